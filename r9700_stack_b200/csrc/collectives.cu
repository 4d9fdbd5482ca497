// Standalone collectives over NVLink / NVSwitch peer memory (pull protocol), for messages the fused
// decode path does not cover: all-reduce (one-shot), all-gather, reduce-scatter; a two-shot
// all-reduce is reduce-scatter followed by all-gather (two calls).
//
// Region of every rank (CUDA IPC shared): [flags: 2 buffers x MAXCH chunks x u32][data: 2 buffers x
// slot_bytes][counters: seq, ticket]. Call g of a collective object uses buffer g & 1 and epoch g + 1:
//   1. every CTA copies its chunk of the input into this rank's own buffer and raises its chunk flag
//      (system-scope fence + release store) -- in its own region: peers pull;
//   2. it waits (bounded, acquire loads over NVLink) for the same chunk's flag of every peer it needs,
//   3. reads the peers' chunks and reduces them in rank order in fp32 (bit-identical on every rank) or
//      gathers them;
//   4. the last CTA to finish (ticket) advances the device sequence counter, so the next launch of
//      the same object -- eager or replayed from a CUDA graph -- uses the next epoch.
// Reuse is safe with two buffers: a rank writes buffer b again at call g + 2 only after passing
// call g + 1, whose flags every peer raised after it had finished reading call g.
// (reference: kernels/r9k_ar.hip:304-358 one-shot N-rank, :370-453 all-gather, :526-639 two-shot,
// with their device seq counters and fixed grids; PCIe there, NVLink here.)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "comm.cuh"

namespace r9k {

constexpr int COLL_MAXCH = 16384;         // chunks per buffer
constexpr int COLL_CHUNK = 4096;          // bf16 elements per chunk (8 KB)
constexpr int64_t COLL_FLAG_BYTES = 2 * COLL_MAXCH * 4;

struct CollArgs {
  uint8_t* base[AR_MAX_WORLD];
  int rank, world;
  int64_t slot_bytes;
  uint32_t* seq;     // this rank's [seq, ticket]
  int* status;
  uint64_t timeout_ns;
};

R9K_DEVINL uint32_t* coll_flag(uint8_t* base, int b, int c) {
  return reinterpret_cast<uint32_t*>(base) + b * COLL_MAXCH + c;
}
R9K_DEVINL __nv_bfloat16* coll_data(uint8_t* base, int b, int64_t slot_bytes) {
  return reinterpret_cast<__nv_bfloat16*>(base + COLL_FLAG_BYTES + b * slot_bytes);
}

// mode 0: all-reduce (out[n] = sum_p x_p)      grid = chunks of n
// mode 1: all-gather (out[p * n + i] = x_p[i])  grid = chunks of n
// mode 2: reduce-scatter (out[i] = sum_p x_p[rank * n / W + i]); grid = chunks of n, CTAs outside
//         this rank's segment only publish their chunk
// vec: every 8-element group of x, out and the peers' slots starts on a 16-byte boundary (checked by
// the host from the pointers and, for the all-gather's rank-major output, n % 8 == 0); otherwise the
// element-wise path runs.
__global__ void __launch_bounds__(256) symm_collective_kernel(CollArgs a, int mode, const __nv_bfloat16* __restrict__ x,
                                                              __nv_bfloat16* __restrict__ out, int64_t n, int vec) {
  pdl_wait();
  pdl_trigger();
  __shared__ int s_ok, s_last;
  __shared__ uint8_t* s_base[AR_MAX_WORLD];  // region bases, indexed by a runtime rank without a local copy
  const int c = blockIdx.x, tid = threadIdx.x;
#pragma unroll
  for (int i = 0; i < AR_MAX_WORLD; ++i)
    if (tid == i) s_base[i] = a.base[i];
  __syncthreads();
  const uint32_t seq = a.seq[0];
  const uint32_t epoch = seq + 1u;
  const int b = (int)(seq & 1u);
  const int64_t e0 = (int64_t)c * COLL_CHUNK, e1 = min(n, e0 + COLL_CHUNK);
  // 1. publish this rank's chunk
  __nv_bfloat16* mine = coll_data(s_base[a.rank], b, a.slot_bytes);
  for (int64_t i = e0 + tid * 8; i < e1; i += 256 * 8) {
    if (vec && i + 8 <= e1) *reinterpret_cast<uint4*>(mine + i) = *reinterpret_cast<const uint4*>(x + i);
    else
      for (int64_t k = i; k < min(e1, i + 8); ++k) mine[k] = x[k];
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    st_release_sys(coll_flag(s_base[a.rank], b, c), epoch);
    s_ok = 1;
  }
  const int64_t seg = n / a.world;
  const bool reduce_here = mode != 2 || (e0 >= (int64_t)a.rank * seg && e1 <= (int64_t)(a.rank + 1) * seg);
  // 2. wait for the peers' chunk
  if (reduce_here && tid < a.world && tid != a.rank) {
    const uint32_t* fl = coll_flag(s_base[tid], b, c);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(fl) < epoch) {
      if (globaltimer_ns() - t0 > a.timeout_ns) {
        report_error(a.status, kErrPeerTimeout, 400, tid);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  // 3. reduce / gather
  if (reduce_here && s_ok) {
    if (mode == 1) {
      for (int p = 0; p < a.world; ++p) {
        const __nv_bfloat16* src = coll_data(s_base[p], b, a.slot_bytes);
        for (int64_t i = e0 + tid * 8; i < e1; i += 256 * 8) {
          if (vec && i + 8 <= e1)
            *reinterpret_cast<uint4*>(out + p * n + i) = ld_volatile_u4(reinterpret_cast<const uint4*>(src + i));
          else
            for (int64_t k = i; k < min(e1, i + 8); ++k) out[p * n + k] = src[k];
        }
      }
    } else {
      const int64_t o0 = mode == 2 ? (int64_t)a.rank * seg : 0;
      for (int64_t i = e0 + tid * 8; i < e1; i += 256 * 8) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const int cnt = (int)min((int64_t)8, e1 - i);
        for (int p = 0; p < a.world; ++p) {
          const __nv_bfloat16* src = coll_data(s_base[p], b, a.slot_bytes) + i;
          if (vec && cnt == 8) {
            const uint4 v = ld_volatile_u4(reinterpret_cast<const uint4*>(src));
            const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] += __bfloat162float(e[k]);
          } else {
            for (int k = 0; k < cnt; ++k) acc[k] += __bfloat162float(src[k]);
          }
        }
        for (int k = 0; k < cnt; ++k) out[i - o0 + k] = __float2bfloat16(acc[k]);
      }
    }
  }
  // 4. the last CTA advances the sequence counter
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(&a.seq[1], 1u);
    s_last = (t == gridDim.x - 1) ? 1 : 0;
  }
  __syncthreads();
  if (s_last && tid == 0) {
    a.seq[1] = 0u;
    a.seq[0] = seq + 1u;
  }
}

void symm_collective(int64_t mode, torch::Tensor x, torch::Tensor out, torch::Tensor peers, int64_t rank,
                     int64_t world, int64_t slot_bytes, torch::Tensor seq, torch::Tensor status, double timeout_s) {
  const int64_t n = x.numel();
  if (n == 0) return;
  TORCH_CHECK(x.dtype() == torch::kBFloat16 && x.is_contiguous() && out.is_contiguous(), "symm_collective: bf16 contiguous");
  TORCH_CHECK(n * 2 <= slot_bytes, "symm_collective: message larger than the slot");
  TORCH_CHECK(world >= 1 && world <= AR_MAX_WORLD && peers.numel() >= world, "symm_collective: world");
  const int64_t nchunks = (n + COLL_CHUNK - 1) / COLL_CHUNK;
  TORCH_CHECK(nchunks <= COLL_MAXCH, "symm_collective: too many chunks");
  if (mode == 2) TORCH_CHECK(n % (world * COLL_CHUNK) == 0, "reduce_scatter: n must be a multiple of world x 4096");
  TORCH_CHECK(out.numel() == (mode == 1 ? n * world : mode == 2 ? n / world : n), "symm_collective: out size");
  CollArgs a = {};
  const int64_t* pp = peers.data_ptr<int64_t>();
  for (int i = 0; i < world; ++i) a.base[i] = reinterpret_cast<uint8_t*>(pp[i]);
  a.rank = (int)rank;
  a.world = (int)world;
  a.slot_bytes = slot_bytes;
  a.seq = reinterpret_cast<uint32_t*>(seq.data_ptr());
  a.status = status.data_ptr<int>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  // the peers' slots start 16-byte aligned (the flag area and slot sizes are multiples of 16)
  TORCH_CHECK(slot_bytes % 16 == 0, "symm_collective: slot size must be a multiple of 16 bytes");
  const bool vec = ((reinterpret_cast<uintptr_t>(x.data_ptr()) | reinterpret_cast<uintptr_t>(out.data_ptr())) & 15) == 0 &&
                   (mode != 1 || n % 8 == 0);
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(launch_pdl(symm_collective_kernel, dim3((unsigned)nchunks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
                         a, (int)mode, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                         reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), n, vec ? 1 : 0) == cudaSuccess,
              "symm_collective launch");
}

int64_t symm_collective_region_bytes(int64_t slot_bytes) { return COLL_FLAG_BYTES + 2 * slot_bytes; }

// ------------------------------------------------------------------------------------------------
// Compressed all-reduce (lossy): every 64-element block of the input is rotated by a 64-point
// Walsh-Hadamard transform (orthonormal, 1/8), scaled by a bf16 scale = amax / qmax and coded as
// 4- or 6-bit two's-complement integers; the ranks' codes are summed in the rotated domain in rank
// order in fp32 and rotated back. Every rank reduces the same packed payloads the same way, so the
// output is bit-identical on all ranks (the rank's own contribution goes through its packed form
// too). Wire bytes per 64 elements: 34 (4-bit) or 50 (6-bit) vs 128 for bf16.
//
// Push protocol, persistent grid (identical on every rank, a function of n only): CTA j owns chunks
// j, j + grid, ...; it packs each chunk into shared memory and stores it with 16-byte posted writes
// into source slot `rank` of buffer b of EVERY rank's region, then raises one flag per rank
// (system-scope fence + release store). The reduce side polls only its own region's flags and reads
// only local memory. Buffer reuse: rank p writes buffer b again at call g + 2 only after its CTA j
// passed call g + 1's wait on rank q's CTA j flag, which q raised after its call g kernel completed.
// Payload of one 4096-element chunk: [64 blocks x 8*bits bytes of codes][64 bf16 scales].
// 4-bit block: byte l = code(2l) & 15 | code(2l+1) << 4. 6-bit block: lane l holds the 12-bit pair
// v_l = code(2l) & 63 | (code(2l+1) & 63) << 6; eight lanes pack 96 bits into three words (v_j at bit
// 12j, little-endian).
// phase 1 publishes, phase 2 waits and reduces (and advances the sequence counter), phase 3 both;
// the split phases let one GPU stand in for several ranks with every wait already satisfied.
// (reference: kernels/r9k_ar_wht.hip:4-27 two-rank pack/reduce, kernels/r9k_ar4.hip:1-42 four-rank
// hierarchy with reductions in the rotated domain; here one flat kernel over NVSwitch peers.)

constexpr int WHT_MAX_CTAS = 2048;  // flag index = source rank * WHT_MAX_CTAS + CTA

// One 64-element block per 8 lanes, 8 elements per lane: element 8*l8 + r in register r of lane
// l8 = lane & 7. Butterflies at strides 1, 2, 4 are in-lane, 8, 16, 32 across lanes (xor 1, 2, 4).
R9K_DEVINL void wht64_8(float (&v)[8], int lane) {
#pragma unroll
  for (int s = 1; s < 8; s <<= 1)
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (!(r & s)) {
        const float lo = v[r], hi = v[r | s];
        v[r] = lo + hi;
        v[r | s] = lo - hi;
      }
#pragma unroll
  for (int m = 1; m < 8; m <<= 1) {
    const bool upper = lane & m;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const float p = __shfl_xor_sync(0xffffffffu, v[r], m);
      v[r] = upper ? p - v[r] : v[r] + p;
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) v[r] *= 0.125f;
}

__host__ __device__ constexpr int wht_chunk_bytes(int bits) { return 64 * 8 * bits + 128; }

R9K_DEVINL void st_u4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
R9K_DEVINL uint4 ld_nc_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
R9K_DEVINL void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}

// Pack the 8 codes of this lane into the block's code bytes (code i of a block at bit bits*i).
R9K_DEVINL void wht_pack(uint8_t* blk, int bits, int l8, const int (&q)[8]) {
  if (bits == 4) {
    uint32_t w = 0;
#pragma unroll
    for (int r = 0; r < 8; ++r) w |= (uint32_t)(q[r] & 15) << (4 * r);
    reinterpret_cast<uint32_t*>(blk)[l8] = w;
  } else {
    uint64_t w = 0;
#pragma unroll
    for (int r = 0; r < 8; ++r) w |= (uint64_t)(q[r] & 63) << (6 * r);
    uint16_t* d = reinterpret_cast<uint16_t*>(blk + 6 * l8);
    d[0] = (uint16_t)w;
    d[1] = (uint16_t)(w >> 16);
    d[2] = (uint16_t)(w >> 32);
  }
}
R9K_DEVINL void wht_unpack_acc(const uint8_t* blk, int bits, int l8, float sf, float (&acc)[8]) {
  if (bits == 4) {
    const uint32_t w = reinterpret_cast<const uint32_t*>(blk)[l8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] += (float)(((int)(w << (28 - 4 * r))) >> 28) * sf;
  } else {
    const uint16_t* d = reinterpret_cast<const uint16_t*>(blk + 6 * l8);
    const uint64_t w = (uint64_t)d[0] | ((uint64_t)d[1] << 16) | ((uint64_t)d[2] << 32);
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] += (float)(((int)((uint32_t)(w >> (6 * r)) << 26)) >> 26) * sf;
  }
  // code * scale is exact in fp32 (<= 6 + 8 significant bits), so fused or not the sums match
}

__global__ void __launch_bounds__(256) symm_ar_wht_kernel(CollArgs a, const __nv_bfloat16* __restrict__ x,
                                                          __nv_bfloat16* __restrict__ out, int64_t n, int bits,
                                                          int phase) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t wsm[];  // publish: one chunk; reduce: 2 x world chunks
  __shared__ int s_ok, s_last;
  __shared__ uint8_t* s_base[AR_MAX_WORLD];  // region bases, indexed by a runtime rank without a local copy
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, cta = blockIdx.x;
  const int l8 = lane & 7, sub = lane >> 3;
#pragma unroll
  for (int i = 0; i < AR_MAX_WORLD; ++i)
    if (tid == i) s_base[i] = a.base[i];
  __syncthreads();
  const uint32_t seq = a.seq[0];
  const uint32_t epoch = seq + 1u;
  const int b = (int)(seq & 1u);
  const int cb = wht_chunk_bytes(bits), nv = cb / 16;
  const int code_bytes = 8 * bits;
  const int qmax = (1 << (bits - 1)) - 1;
  const int64_t nchunks = (n + COLL_CHUNK - 1) / COLL_CHUNK;
  const int64_t src_cap = (a.slot_bytes / a.world) & ~(int64_t)15;
  // block of (chunk, iteration it) handled by this lane group: 4 * (warp + 8 * it) + sub
  auto blk_of = [&](int it) { return 4 * (warp + 8 * it) + sub; };
  if (phase & 1) {
    uint4 nxt[2];
    auto load = [&](int64_t c, uint4 (&v)[2]) {
      const int64_t e0 = c * COLL_CHUNK;
#pragma unroll
      for (int it = 0; it < 2; ++it) {
        const int64_t e = e0 + 64 * blk_of(it) + 8 * l8;
        v[it] = (c < nchunks && e < n) ? ld_nc_u4(x + e) : make_uint4(0, 0, 0, 0);
      }
    };
    load(cta, nxt);
    for (int64_t c = cta; c < nchunks; c += gridDim.x) {
      uint4 cur[2] = {nxt[0], nxt[1]};
      load(c + gridDim.x, nxt);  // next chunk's loads in flight while this one is coded
      const int64_t e0 = c * COLL_CHUNK;
      const int nblk = (int)(min(n - e0, (int64_t)COLL_CHUNK) / 64);
#pragma unroll
      for (int it = 0; it < 2; ++it) {
        const int bi = blk_of(it);
        float v[8];
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&cur[it]);
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = __bfloat162float(h[r]);
        wht64_8(v, lane);
        float amax = 0.f;
#pragma unroll
        for (int r = 0; r < 8; ++r) amax = fmaxf(amax, fabsf(v[r]));
#pragma unroll
        for (int m = 1; m < 8; m <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        const __nv_bfloat16 sb = __float2bfloat16(amax / (float)qmax);
        const float sf = __bfloat162float(sb);
        const float inv = sf > 0.f ? 1.f / sf : 0.f;
        int q[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) q[r] = max(-qmax, min(qmax, __float2int_rn(v[r] * inv)));
        if (bi < nblk) {
          wht_pack(wsm + bi * code_bytes, bits, l8, q);
          if (l8 == 0) reinterpret_cast<__nv_bfloat16*>(wsm + 64 * code_bytes)[bi] = sb;
        }
      }
      __syncthreads();
      // push the packed chunk into source slot `rank` of every rank's buffer b
      const int nvc = (nblk * code_bytes) / 16, nvs = (nblk * 2 + 15) / 16, s0 = 64 * code_bytes / 16;
      for (int i = tid; i < a.world * nv; i += 256) {
        const int p = i / nv, k = i - p * nv;
        if (k < nvc || (k >= s0 && k < s0 + nvs)) {
          uint8_t* dst = reinterpret_cast<uint8_t*>(coll_data(s_base[p], b, a.slot_bytes)) + a.rank * src_cap + c * cb;
          st_u4(dst + 16 * k, reinterpret_cast<const uint4*>(wsm)[k]);
        }
      }
      __syncthreads();
    }
    if (tid == 0) {
      __threadfence_system();
      for (int p = 0; p < a.world; ++p) st_release_sys(coll_flag(s_base[p], b, a.rank * WHT_MAX_CTAS + cta), epoch);
    }
  }
  if (!(phase & 2)) return;
  if (tid == 0) s_ok = 1;
  __syncthreads();
  if (tid < a.world && tid != a.rank) {
    const uint32_t* fl = coll_flag(s_base[a.rank], b, tid * WHT_MAX_CTAS + cta);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(fl) < epoch) {
      if (globaltimer_ns() - t0 > a.timeout_ns) {
        report_error(a.status, kErrPeerTimeout, 401, tid);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (s_ok) {
    const uint8_t* mine = reinterpret_cast<const uint8_t*>(coll_data(s_base[a.rank], b, a.slot_bytes));
    const int wcb = a.world * cb;
    auto fetch = [&](int64_t c, int buf) {
      if (c < nchunks)
        for (int i = tid; i < a.world * nv; i += 256) {
          const int p = i / nv, k = i - p * nv;
          cp_async16(wsm + buf * wcb + p * cb + 16 * k, mine + p * src_cap + c * cb + 16 * k);
        }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    fetch(cta, 0);
    int buf = 0;
    for (int64_t c = cta; c < nchunks; c += gridDim.x, buf ^= 1) {
      fetch(c + gridDim.x, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
      __syncthreads();
      const int64_t e0 = c * COLL_CHUNK;
      const int nblk = (int)(min(n - e0, (int64_t)COLL_CHUNK) / 64);
#pragma unroll
      for (int it = 0; it < 2; ++it) {
        const int bi = blk_of(it);  // groups past the end compute on stale bytes and store nothing
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int p = 0; p < a.world; ++p) {
          const uint8_t* pl = wsm + buf * wcb + p * cb;
          const float sf = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(pl + 64 * code_bytes)[bi]);
          wht_unpack_acc(pl + bi * code_bytes, bits, l8, sf, acc);
        }
        wht64_8(acc, lane);
        uint4 o;
        __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int r = 0; r < 4; ++r) ob[r] = __floats2bfloat162_rn(acc[2 * r], acc[2 * r + 1]);
        if (bi < nblk) *reinterpret_cast<uint4*>(out + e0 + 64 * bi + 8 * l8) = o;
      }
      __syncthreads();
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(&a.seq[1], 1u);
    s_last = (t == gridDim.x - 1) ? 1 : 0;
  }
  __syncthreads();
  if (s_last && tid == 0) {
    a.seq[1] = 0u;
    a.seq[0] = seq + 1u;
  }
}

void symm_ar_wht(torch::Tensor x, torch::Tensor out, torch::Tensor peers, int64_t rank, int64_t world,
                 int64_t slot_bytes, torch::Tensor seq, torch::Tensor status, double timeout_s, int64_t bits,
                 int64_t phase) {
  const int64_t n = x.numel();
  if (n == 0) return;
  TORCH_CHECK(bits == 4 || bits == 6, "symm_ar_wht: bits must be 4 or 6");
  TORCH_CHECK(phase >= 1 && phase <= 3, "symm_ar_wht: phase 1 (publish), 2 (reduce) or 3 (both)");
  TORCH_CHECK(x.dtype() == torch::kBFloat16 && out.dtype() == torch::kBFloat16 && x.is_contiguous() &&
                  out.is_contiguous() && out.numel() == n,
              "symm_ar_wht: bf16 contiguous x and out of the same size");
  TORCH_CHECK(n % 64 == 0, "symm_ar_wht: size must be a multiple of 64");
  TORCH_CHECK(((reinterpret_cast<uintptr_t>(x.data_ptr()) | reinterpret_cast<uintptr_t>(out.data_ptr())) & 3) == 0,
              "symm_ar_wht: x and out must be 4-byte aligned");
  TORCH_CHECK(world >= 1 && world <= AR_MAX_WORLD && peers.numel() >= world, "symm_ar_wht: world");
  const int64_t nchunks = (n + COLL_CHUNK - 1) / COLL_CHUNK;
  TORCH_CHECK(nchunks * wht_chunk_bytes((int)bits) <= ((slot_bytes / world) & ~(int64_t)15),
              "symm_ar_wht: message larger than the slot (world x payload)");
  TORCH_CHECK(slot_bytes % 16 == 0, "symm_ar_wht: slot size must be a multiple of 16 bytes");
  CollArgs a = {};
  const int64_t* pp = peers.data_ptr<int64_t>();
  for (int i = 0; i < world; ++i) a.base[i] = reinterpret_cast<uint8_t*>(pp[i]);
  a.rank = (int)rank;
  a.world = (int)world;
  a.slot_bytes = slot_bytes;
  a.seq = reinterpret_cast<uint32_t*>(seq.data_ptr());
  a.status = status.data_ptr<int>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(((reinterpret_cast<uintptr_t>(x.data_ptr()) | reinterpret_cast<uintptr_t>(out.data_ptr())) & 15) == 0,
              "symm_ar_wht: x and out must be 16-byte aligned");
  const int smem = 2 * (int)world * wht_chunk_bytes((int)bits);
  // persistent grid: four CTAs per SM, a function of n only (identical on every rank)
  const int grid = (int)std::min<int64_t>(nchunks, 4 * 148);
  static_assert(4 * 148 <= WHT_MAX_CTAS && AR_MAX_WORLD * WHT_MAX_CTAS <= COLL_MAXCH, "flag table");
  TORCH_CHECK(ensure_smem_attr((const void*)symm_ar_wht_kernel, 2 * AR_MAX_WORLD * wht_chunk_bytes(6)) == cudaSuccess,
              "symm_ar_wht smem attribute");
  TORCH_CHECK(launch_pdl(symm_ar_wht_kernel, dim3((unsigned)grid), dim3(256), smem, at::cuda::getCurrentCUDAStream(), a,
                         reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                         reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), n, (int)bits, (int)phase) == cudaSuccess,
              "symm_ar_wht launch");
}

}  // namespace r9k
