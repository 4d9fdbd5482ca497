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

constexpr int COLL_MAXCH = 4096;          // chunks per buffer
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
  const int c = blockIdx.x, tid = threadIdx.x;
  const uint32_t seq = a.seq[0];
  const uint32_t epoch = seq + 1u;
  const int b = (int)(seq & 1u);
  const int64_t e0 = (int64_t)c * COLL_CHUNK, e1 = min(n, e0 + COLL_CHUNK);
  // 1. publish this rank's chunk
  __nv_bfloat16* mine = coll_data(a.base[a.rank], b, a.slot_bytes);
  for (int64_t i = e0 + tid * 8; i < e1; i += 256 * 8) {
    if (vec && i + 8 <= e1) *reinterpret_cast<uint4*>(mine + i) = *reinterpret_cast<const uint4*>(x + i);
    else
      for (int64_t k = i; k < min(e1, i + 8); ++k) mine[k] = x[k];
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    st_release_sys(coll_flag(a.base[a.rank], b, c), epoch);
    s_ok = 1;
  }
  const int64_t seg = n / a.world;
  const bool reduce_here = mode != 2 || (e0 >= (int64_t)a.rank * seg && e1 <= (int64_t)(a.rank + 1) * seg);
  // 2. wait for the peers' chunk
  if (reduce_here && tid < a.world && tid != a.rank) {
    const uint32_t* fl = coll_flag(a.base[tid], b, c);
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
        const __nv_bfloat16* src = coll_data(a.base[p], b, a.slot_bytes);
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
          const __nv_bfloat16* src = coll_data(a.base[p], b, a.slot_bytes) + i;
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

}  // namespace r9k
