// NVLink SHARP (NVLS) collectives over a multicast mapping of symmetric buffers.
//
// The buffers come from torch's symmetric memory (one allocation per rank, mapped into every peer and
// bound to one NVSwitch multicast object); `mc` addresses all ranks' copies at once:
//   multimem.ld_reduce  reads the same offset on every GPU and returns the sum, reduced in the switch;
//   multimem.st         writes one value to the same offset on every GPU.
// Two-shot all-reduce, one kernel: every CTA c
//   1. copies its part of every slice of the input into this rank's buffer,
//   2. barrier with CTA c of every peer (all inputs of part c are in place),
//   3. reduces part c of this rank's slice with ld_reduce (fp32 accumulation in the switch) and
//      broadcasts the bf16 result with multimem.st -- every element is reduced once, by its owner, so
//      every rank ends with the same bits,
//   4. barrier again (every owner's broadcast of part c landed here),
//   5. copies part c of every slice from the buffer to the output.
// The all-gather writes each rank's input straight to its offset of every copy with multimem.st.
// Barriers: thread q of CTA c release-stores the call's epoch into slot (c, rank) of peer q's signal
// pad and acquire-polls slot (c, q) of its own pad (bounded; a timeout writes the status word). The
// epoch comes from a device sequence counter that the last CTA advances, so the kernel replays inside
// CUDA graphs. Buffer reuse is safe: a rank overwrites part c of its buffer in the next call only
// after passing this call's second barrier, which every peer's CTA c reached after its reduction.
// Reference: kernels/r9k_ar.hip:526-639 (two-shot all-reduce over PCIe P2P); here the switch reduces.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "comm.cuh"

namespace r9k {

constexpr int NVLS_MAX_CTAS = 256;

struct NvlsArgs {
  uint8_t* mc;                     // multicast address of the symmetric buffer
  uint8_t* local;                  // this rank's copy
  uint32_t* sig[AR_MAX_WORLD];     // every rank's signal pad
  int rank, world;
  uint32_t* seq;                   // this object's [sequence, ticket] counters (device)
  int* status;
  uint64_t timeout_ns;
};

R9K_DEVINL uint4 mm_ld_reduce_bf16x8(const void* p) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p) : "memory");
  return r;
}
R9K_DEVINL void mm_st_v4(void* p, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w) : "memory");
}

// CTA-wide barrier with CTA `slot` of every rank; false if a peer did not arrive in time
// (epochs only grow: every collective on one signal pad draws them from the same sequence counter)
R9K_DEVINL bool nvls_barrier(const NvlsArgs& a, int slot, uint32_t epoch) {
  // multicast stores and the unicast reads after the barrier reach the same memory through two
  // virtual aliases
  asm volatile("fence.proxy.alias;" ::: "memory");
  __syncthreads();  // every thread's stores of this CTA happen before the release below
  bool ok = true;
  if (threadIdx.x < a.world) {
    const int q = threadIdx.x;
    st_release_sys(a.sig[q] + slot * AR_MAX_WORLD + a.rank, epoch);
    const uint32_t* f = a.sig[a.rank] + slot * AR_MAX_WORLD + q;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(f) < epoch) {
      if (globaltimer_ns() - t0 > a.timeout_ns) {
        report_error(a.status, kErrPeerTimeout, 400, slot * 256 + q);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

R9K_DEVINL void nvls_ticket(const NvlsArgs& a, uint32_t seq) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(&a.seq[1], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    a.seq[1] = 0u;
    a.seq[0] = seq + 1u;
  }
}

// n elements (bf16), n % (8 * world) == 0; grid = C CTAs, part = ceil(per_rank / 8 / C) vectors
__global__ void __launch_bounds__(512) nvls_allreduce_kernel(NvlsArgs a, const __nv_bfloat16* __restrict__ x,
                                                             __nv_bfloat16* __restrict__ out, int64_t n, int copy_in) {
  pdl_wait();
  const uint32_t seq = a.seq[0];
  const int c = blockIdx.x, C = gridDim.x, W = a.world;
  const int64_t per = n / W / 8;                 // 16-byte vectors per slice
  const int64_t part = (per + C - 1) / C;
  const int64_t v0 = (int64_t)c * part, v1 = min(per, v0 + part);
  uint4* loc = reinterpret_cast<uint4*>(a.local);
  if (copy_in) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int s = 0; s < W; ++s)
      for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) loc[s * per + i] = xv[s * per + i];
  }
  if (!nvls_barrier(a, c, 2 * seq + 1)) return;
  uint4* mcv = reinterpret_cast<uint4*>(a.mc);
  for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
    const int64_t o = (int64_t)a.rank * per + i;
    mm_st_v4(mcv + o, mm_ld_reduce_bf16x8(mcv + o));
  }
  if (!nvls_barrier(a, c, 2 * seq + 2)) return;
  pdl_trigger();
  uint4* ov = reinterpret_cast<uint4*>(out);
  for (int s = 0; s < W; ++s)
    for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) ov[s * per + i] = loc[s * per + i];
  nvls_ticket(a, seq);
}

// all-gather: out [W, n] = every rank's x [n] (4-byte elements as raw words), n * 4 % 16 == 0
__global__ void __launch_bounds__(512) nvls_allgather_kernel(NvlsArgs a, const uint4* __restrict__ x,
                                                             uint4* __restrict__ out, int64_t nvec) {
  pdl_wait();
  const uint32_t seq = a.seq[0];
  const int c = blockIdx.x, C = gridDim.x, W = a.world;
  const int64_t part = (nvec + C - 1) / C;
  const int64_t v0 = (int64_t)c * part, v1 = min(nvec, v0 + part);
  uint4* mcv = reinterpret_cast<uint4*>(a.mc);
  for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) mm_st_v4(mcv + (int64_t)a.rank * nvec + i, x[i]);
  if (!nvls_barrier(a, c, 2 * seq + 1)) return;
  pdl_trigger();
  const uint4* loc = reinterpret_cast<const uint4*>(a.local);
  for (int s = 0; s < W; ++s)
    for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) out[s * nvec + i] = loc[s * nvec + i];
  // second barrier: no rank overwrites its copy in the next call while a peer still reads it here
  if (!nvls_barrier(a, c, 2 * seq + 2)) return;
  nvls_ticket(a, seq);
}

static NvlsArgs nvls_args(int64_t mc, int64_t local, torch::Tensor sig_ptrs, int64_t rank, int64_t world,
                          torch::Tensor seq, torch::Tensor status, double timeout_s) {
  TORCH_CHECK(world >= 1 && world <= AR_MAX_WORLD, "nvls: world 1..8");
  TORCH_CHECK(sig_ptrs.device().is_cpu() && sig_ptrs.dtype() == torch::kInt64 && sig_ptrs.numel() >= world,
              "nvls: CPU int64 signal-pad table");
  TORCH_CHECK(mc != 0 && local != 0, "nvls: multicast and local buffer addresses");
  NvlsArgs a = {};
  a.mc = reinterpret_cast<uint8_t*>(mc);
  a.local = reinterpret_cast<uint8_t*>(local);
  for (int i = 0; i < world; ++i) a.sig[i] = reinterpret_cast<uint32_t*>(sig_ptrs.data_ptr<int64_t>()[i]);
  a.rank = (int)rank;
  a.world = (int)world;
  a.seq = reinterpret_cast<uint32_t*>(seq.data_ptr());
  a.status = status.data_ptr<int>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  return a;
}

static int nvls_ctas(int64_t vecs_per_cta_side, int64_t nvec) {
  int64_t C = (nvec + vecs_per_cta_side - 1) / vecs_per_cta_side;
  return (int)std::max<int64_t>(1, std::min<int64_t>(NVLS_MAX_CTAS, C));
}

// x: bf16 [n] (or already in the local buffer when x is null); out: bf16 [n]
void nvls_all_reduce(c10::optional<torch::Tensor> x, torch::Tensor out, int64_t mc, int64_t local, int64_t cap_bytes,
                     torch::Tensor sig_ptrs, int64_t sig_slots, int64_t rank, int64_t world, torch::Tensor seq,
                     torch::Tensor status, double timeout_s) {
  const int64_t n = out.numel();
  TORCH_CHECK(out.dtype() == torch::kBFloat16 && out.is_contiguous(), "nvls_all_reduce: bf16 contiguous out");
  TORCH_CHECK(n % (8 * world) == 0 && n * 2 <= cap_bytes, "nvls_all_reduce: n % (8 world) and capacity");
  const bool copy_in = x.has_value() && x->defined();
  if (copy_in) TORCH_CHECK(x->numel() == n && x->dtype() == torch::kBFloat16 && x->is_contiguous(), "nvls_all_reduce: x");
  TORCH_CHECK(((reinterpret_cast<uintptr_t>(out.data_ptr()) |
                (copy_in ? reinterpret_cast<uintptr_t>(x->data_ptr()) : 0)) & 15) == 0, "nvls_all_reduce: 16-byte aligned");
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(out.device());
  NvlsArgs a = nvls_args(mc, local, sig_ptrs, rank, world, seq, status, timeout_s);
  const int C = std::min<int>(nvls_ctas(4096, n / world / 8), (int)(sig_slots / AR_MAX_WORLD));
  TORCH_CHECK(launch_pdl(nvls_allreduce_kernel, dim3((unsigned)C), dim3(512), 0, at::cuda::getCurrentCUDAStream(), a,
                         copy_in ? reinterpret_cast<const __nv_bfloat16*>(x->data_ptr()) : nullptr,
                         reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), n, copy_in ? 1 : 0) == cudaSuccess,
              "nvls_all_reduce launch");
}

// x: [R, m] (4-byte elements) -> out [W, R, m] (rank-major)
void nvls_all_gather(torch::Tensor x, torch::Tensor out, int64_t mc, int64_t local, int64_t cap_bytes,
                     torch::Tensor sig_ptrs, int64_t sig_slots, int64_t rank, int64_t world, torch::Tensor seq,
                     torch::Tensor status, double timeout_s) {
  const int64_t bytes = x.numel() * x.element_size();
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && out.numel() == x.numel() * world, "nvls_all_gather: shapes");
  TORCH_CHECK(bytes % 16 == 0 && bytes * world <= cap_bytes, "nvls_all_gather: 16-byte multiple and capacity");
  TORCH_CHECK(((reinterpret_cast<uintptr_t>(x.data_ptr()) | reinterpret_cast<uintptr_t>(out.data_ptr())) & 15) == 0,
              "nvls_all_gather: 16-byte aligned");
  if (bytes == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  NvlsArgs a = nvls_args(mc, local, sig_ptrs, rank, world, seq, status, timeout_s);
  const int64_t nvec = bytes / 16;
  const int C = std::min<int>(nvls_ctas(2048, nvec), (int)(sig_slots / AR_MAX_WORLD));
  TORCH_CHECK(launch_pdl(nvls_allgather_kernel, dim3((unsigned)C), dim3(512), 0, at::cuda::getCurrentCUDAStream(), a,
                         reinterpret_cast<const uint4*>(x.data_ptr()), reinterpret_cast<uint4*>(out.data_ptr()), nvec) ==
                  cudaSuccess,
              "nvls_all_gather launch");
}

}  // namespace r9k
