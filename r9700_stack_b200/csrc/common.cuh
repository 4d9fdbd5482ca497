// Shared device helpers for the sm_100a kernels: mbarriers, TMA, tcgen05 (TMEM alloc, MMA,
// commit, ld, cp), UMMA descriptors, bounded waits and the status word.
//
// Every spin in this library is bounded by a %globaltimer deadline. A wait that gives up writes
// an error record into the caller's status buffer and the kernel returns; no kernel traps.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <mutex>
#include <set>
#include <utility>

#define R9K_DEVINL __device__ __forceinline__

namespace r9k {

// ---------------------------------------------------------------------------------------------
// status word: [0] = error code (0 ok), [1] = kernel id, [2] = block, [3] = detail
// ---------------------------------------------------------------------------------------------
enum : int {
  kErrNone = 0,
  kErrMbarTimeout = 1,
  kErrPeerTimeout = 2,
  kErrBounds = 3,
  kErrConfig = 4,
};

R9K_DEVINL void report_error(int* status, int code, int kernel_id, int detail) {
  if (status == nullptr) return;
  if (atomicCAS(status, 0, code) == 0) {
    status[1] = kernel_id;
    status[2] = (int)(blockIdx.x + blockIdx.y * gridDim.x);
    status[3] = detail;
  }
}

R9K_DEVINL uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

R9K_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

R9K_DEVINL uint32_t lane_id() { return threadIdx.x & 31; }
R9K_DEVINL uint32_t warp_id() { return threadIdx.x >> 5; }

R9K_DEVINL bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------------------------
// programmatic dependent launch: a kernel launched with the programmatic-serialization attribute may
// start before its predecessor finishes; it must call pdl_wait() before touching anything the
// predecessor writes (or reads). pdl_trigger() lets the successor launch early.
// ---------------------------------------------------------------------------------------------
R9K_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
R9K_DEVINL void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with programmatic stream serialisation (the kernel must pdl_wait() before it touches
// memory its predecessor writes or reads). Launch errors are returned to the caller's check.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Set a kernel's dynamic shared-memory limit once per (kernel, device). The attribute belongs to the
// device's context, so a process that drives several GPUs needs it set on each of them.
inline cudaError_t ensure_smem_attr(const void* kern, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({kern, dev})) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert({kern, dev});
  return e;
}

// The multiprocessor count of the current device (cached per device).
inline int device_sm_count() {
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
R9K_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
R9K_DEVINL void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
R9K_DEVINL void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
R9K_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
R9K_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
R9K_DEVINL bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded parity wait. Returns false when the deadline passes (the caller reports and bails).
R9K_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(addr, parity)) return true;
    if (globaltimer_ns() - t0 > timeout_ns) return false;
  }
}

// ---------------------------------------------------------------------------------------------
// TMA / bulk copies (no cluster multicast anywhere in this library)
// ---------------------------------------------------------------------------------------------
R9K_DEVINL void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
R9K_DEVINL void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                 uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(hint)
      : "memory");
}
R9K_DEVINL void tma_load_3d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                 uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(hint)
      : "memory");
}
// L2 prefetch of a tensor-map tile (no shared memory, no barrier): warms L2 for a later TMA load of the
// same coordinates. Not a multicast load.
R9K_DEVINL void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
R9K_DEVINL void tma_prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}
R9K_DEVINL void bulk_prefetch_l2(const void* gsrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}
// Plain bulk copy global -> shared (16-byte aligned addresses, size multiple of 16).
R9K_DEVINL void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
R9K_DEVINL void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// L2 eviction policies for cache hints
R9K_DEVINL uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
R9K_DEVINL uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads, smem->tmem copies
// ---------------------------------------------------------------------------------------------
R9K_DEVINL void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
R9K_DEVINL void tmem_relinquish() {  // whole warp
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
R9K_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
R9K_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
R9K_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16/f16 inputs, f32 accumulate)
R9K_DEVINL void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}
// kind::f8f6f4 (unscaled fp8/fp6/fp4 inputs)
R9K_DEVINL void mma_f8f6f4_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                              uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}
// kind::mxf8f6f4 with ue8m0 block-32 scale factors held in TMEM
R9K_DEVINL void mma_mxf8f6f4_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                uint32_t accum, uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// Arrive on an mbarrier when all previously issued tcgen05 ops of this thread complete.
R9K_DEVINL void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// smem (32 rows x 16 B) -> TMEM, replicated into all four 32-lane sub-partitions
R9K_DEVINL void tc_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
R9K_DEVINL void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns -> 16 registers per thread
R9K_DEVINL void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
R9K_DEVINL void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 lanes x 32 bit store, 16 columns (used to seed TMEM, e.g. P tiles)
R9K_DEVINL void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
R9K_DEVINL void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------------------------
// K-major operand tile written by TMA with SWIZZLE_128B: rows of 128 bytes, 8-row groups of 1 KiB.
// Fields: start>>4 [0,14), LBO>>4 [16,30) (unused for swizzled K-major, set to 1), SBO>>4 [32,46),
// version 1 at bit 46, layout type at [61,64) (2 = 128B swizzle).
R9K_DEVINL uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}
// Scale-factor block for tcgen05.cp 32x128b: 32 rows of 16 bytes, contiguous, no swizzle.
// 8-row core matrices are 128 bytes apart (SBO); one core matrix along K (LBO unused).
R9K_DEVINL uint64_t sdesc_sf(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(128u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// Instruction descriptor, kind::f16 / kind::f8f6f4 (dense):
//  [4,6) c_format (1 = f32), [7,10) a_format, [10,13) b_format, [15] a_major, [16] b_major,
//  [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t idesc_dense(uint32_t a_fmt, uint32_t b_fmt, int M, int N) {
  return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Instruction descriptor, block-scaled kinds:
//  [4,6) b_sf_id, [7,10) a_format, [10,13) b_format, [17,23) N>>3, [23] scale format (1 = ue8m0),
//  [24,29) M>>4, [29,31) a_sf_id.
__host__ __device__ constexpr uint32_t idesc_block_scaled(uint32_t a_fmt, uint32_t b_fmt, int M, int N,
                                                          uint32_t a_sf_id, uint32_t b_sf_id) {
  return (b_sf_id << 4) | (a_fmt << 7) | (b_fmt << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(M >> 4) << 24) | (a_sf_id << 29);
}
enum : uint32_t {
  kFmtF16 = 0, kFmtBF16 = 1,                      // kind::f16
  kFmtE4M3 = 0, kFmtE5M2 = 1, kFmtE2M1 = 5,        // kind::f8f6f4 / mxf8f6f4
};

// ---------------------------------------------------------------------------------------------
// cluster helpers (distributed shared memory)
// ---------------------------------------------------------------------------------------------
R9K_DEVINL uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
R9K_DEVINL uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
R9K_DEVINL void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// map a local shared address to the same offset in CTA `rank` of the cluster
R9K_DEVINL uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
R9K_DEVINL float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// ---------------------------------------------------------------------------------------------
// numerics
// ---------------------------------------------------------------------------------------------
R9K_DEVINL float silu_f(float x) { return x / (1.0f + __expf(-x)); }
R9K_DEVINL float sigmoid_f(float x) { return 1.0f / (1.0f + __expf(-x)); }
R9K_DEVINL float softplus_f(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// ue8m0 exponent for an MX block so that amax / 2^e <= qmax:  e = ceil(log2(amax / qmax)).
// Computed exactly from the float bits (no transcendental): for r = amax/qmax in normal range,
// ceil(log2 r) = unbiased exponent of r, plus one if r has a non-zero mantissa.
R9K_DEVINL int mx_exponent(float amax, float qmax) {
  if (!(amax > 0.f)) return -127;
  float r = amax / qmax;
  uint32_t b = __float_as_uint(r);
  int e = (int)((b >> 23) & 0xff) - 127;
  if (((b >> 23) & 0xff) == 0) return -127;  // subnormal ratio: smallest scale
  if (b & 0x7fffff) e += 1;
  return max(-127, min(127, e));
}
R9K_DEVINL float exp2i(int e) {  // 2^e for e in [-126, 127] exactly
  return __uint_as_float((uint32_t)(e + 127) << 23);
}
R9K_DEVINL uint8_t f32_to_e4m3(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
R9K_DEVINL float e4m3_to_f32(uint8_t v) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)v, __NV_E4M3);
  return __half2float(__half(h));
}

// Offset of the ue8m0 scale byte for (row, k-block) inside the 512-byte scale chunks the MMA
// consumes: chunks are ordered [row / 128][k-block / 4]; inside a chunk the byte for row r and
// k-block j sits at (r % 32) * 16 + ((r % 128) / 32) * 4 + (j % 4).
__host__ __device__ inline int64_t sf_offset(int64_t row, int64_t kblk, int64_t kblocks_total) {
  const int64_t kchunks = (kblocks_total + 3) / 4;
  const int64_t chunk = (row >> 7) * kchunks + (kblk >> 2);
  return chunk * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 + (kblk & 3);
}

}  // namespace r9k
