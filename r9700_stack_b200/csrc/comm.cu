// Tensor-parallel communication over NVLink / NVSwitch peer memory.
//
// Symmetric buffers: each rank cudaMalloc's one region and shares it with its peers through CUDA IPC
// handles (exchanged on the host); every rank then holds device pointers to all peers' regions.
//
// Fused all-reduce (decode path):
//   producer  - the row-parallel GEMM (o_proj / out_proj / down_proj) epilogue, or push_partial for
//               other producers, writes its bf16 partial [T, H] into slot [src rank] of every rank's
//               region (P2P stores over NVLink) and then raises, per 128-column tile, a flag word
//               (fence.acq_rel.sys + st.release.sys) holding the call's epoch.
//   consumer  - ar_rmsnorm: per token row, waits (bounded, acquire loads) for the flags of every
//               tile from every rank, sums the ranks' partials in rank order in fp32 (so all ranks
//               get bit-identical results), adds the residual, applies RMSNorm and writes the new
//               residual plus MXFP8 (or bf16) input of the next GEMM.
// Epochs: a device-resident step counter (bumped once per model step by step_begin) and the call's
// static index k within the step give the global call g = step * calls_per_step + k (calls_per_step
// even), epoch g + 1 and buffer g % 2. A rank can only write call g+2's data after every rank
// finished reading call g (it needed their call g+1 flags, raised after their call g consumer), so
// two alternating buffers suffice and the scheme replays inside CUDA graphs. Reference counterpart: r9k_ar_oneshot_nrank + double-buffered device
// seq counters, kernels/r9k_ar.hip:12-48, :304-358 (PCIe P2P); here the reduction is fused into the
// producing GEMM and the consuming norm.
//
// Waits give up after a deadline and record {code, kernel, block, detail} in the status word.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "comm.cuh"

namespace r9k {

// ------------------------------------------------------------------------------------------------
// host: symmetric regions through CUDA IPC
// ------------------------------------------------------------------------------------------------
int64_t symm_alloc(int64_t nbytes) {
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, (size_t)nbytes) == cudaSuccess, "symm_alloc: cudaMalloc failed");
  TORCH_CHECK(cudaMemset(p, 0, (size_t)nbytes) == cudaSuccess, "symm_alloc: memset failed");
  TORCH_CHECK(cudaDeviceSynchronize() == cudaSuccess, "symm_alloc: sync failed");
  return reinterpret_cast<int64_t>(p);
}

void symm_free(int64_t ptr) { cudaFree(reinterpret_cast<void*>(ptr)); }

torch::Tensor symm_ipc_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)) == cudaSuccess, "cudaIpcGetMemHandle failed");
  auto t = torch::empty({(int64_t)sizeof(h)}, torch::dtype(torch::kUInt8));
  memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t symm_open(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "symm_open: bad handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  TORCH_CHECK(e == cudaSuccess, "cudaIpcOpenMemHandle failed: ", cudaGetErrorString(e));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

// a bf16 [rows, cols] view of device memory at ptr (for tests and local reads)
torch::Tensor symm_view(int64_t ptr, int64_t offset_bytes, int64_t rows, int64_t cols, int64_t device) {
  auto opts = torch::dtype(torch::kBFloat16).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<uint8_t*>(ptr) + offset_bytes, {rows, cols}, opts);
}

// ------------------------------------------------------------------------------------------------
// kernels
// ------------------------------------------------------------------------------------------------
__global__ void step_begin_kernel(uint32_t* step) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  if (threadIdx.x == 0) step[0] = step[0] + 1;
}

void symm_step_begin(torch::Tensor step) {
  launch_pdl(step_begin_kernel, dim3(1), dim3(32), 0, at::cuda::getCurrentCUDAStream(),reinterpret_cast<uint32_t*>(step.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// standalone producer: push x [T, H] (bf16) into every rank's slot and raise the tile flags
__global__ void push_partial_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, ArPeers pe, int T, int H,
                                    int call) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  const ArCall arc = ar_resolve(pe, call);
  const int tile = blockIdx.x;  // 128-column tile
  const int c0 = tile * 128;
  for (int t = threadIdx.y; t < T; t += blockDim.y) {
    const int c = c0 + threadIdx.x * 4;
    if (c >= H) continue;
    const uint2 v = *reinterpret_cast<const uint2*>(x + (int64_t)t * ldx + c);
#pragma unroll
    for (int p = 0; p < AR_MAX_WORLD; ++p)
      if (p < pe.world) *reinterpret_cast<uint2*>(arc.dst[p] + (int64_t)t * H + c) = v;
  }
  __syncthreads();
  if (threadIdx.x == 0 && threadIdx.y == 0) ar_raise_flags(pe, call, tile, arc.epoch);
}

void push_partial(torch::Tensor x, torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems,
                  int64_t call, torch::Tensor step, int64_t calls_per_step) {
  const int64_t T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 128 == 0 && T * H <= slot_elems, "push_partial: H % 128 and T*H within the slot");
  const at::cuda::CUDAGuard guard(x.device());
  ArPeers pe = make_peers(peers, rank, world, slot_elems, H, step, calls_per_step);
  launch_pdl(push_partial_kernel, dim3((unsigned)(H / 128)), dim3(32, 8), 0, at::cuda::getCurrentCUDAStream(),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), pe, (int)T, (int)H, (int)call);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// consumer: all-reduce (rank order) + residual add + RMSNorm (+ MXFP8). One CTA per token row,
// one thread per 32-element block.
__global__ void ar_rmsnorm_kernel(ArPeers pe, int call, const __nv_bfloat16* __restrict__ res_in,
                                  __nv_bfloat16* __restrict__ res_out, const __nv_bfloat16* __restrict__ w, int K,
                                  float eps, int plus_one, __nv_bfloat16* __restrict__ y, uint8_t* __restrict__ q,
                                  uint8_t* __restrict__ sf, int* status, uint64_t timeout_ns) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  __shared__ float sred[32];
  __shared__ int s_fail;
  const int64_t r = blockIdx.x;
  const int kblocks = K / 32;
  const int blk = threadIdx.x;
  const uint32_t gcall = ar_global_call(pe, call);
  const uint32_t epoch = gcall + 1u;
  const uint32_t buf = gcall & 1u;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  // wait for every (rank, tile) flag of this call: thread i polls flags i, i + blockDim, ...
  const int ntiles = K / 128;
  const uint64_t t0 = globaltimer_ns();
  for (int f = threadIdx.x; f < pe.world * ntiles; f += blockDim.x) {
    const int src = f / ntiles, tile = f % ntiles;
    const uint32_t* fl = reinterpret_cast<const uint32_t*>(pe.base[pe.rank]) +
                         ((int64_t)buf * AR_MAX_WORLD + src) * AR_MAX_TILES + tile;
    while (ld_acquire_sys(fl) < epoch) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        s_fail = 1;
        report_error(status, kErrPeerTimeout, 300, src * 65536 + tile);
        break;
      }
    }
  }
  __syncthreads();
  const bool act = blk < kblocks && !s_fail;
  float v[32];
  float ss = 0.f;
  if (act) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
    for (int src = 0; src < pe.world; ++src) {  // fixed rank order: identical sums on every rank
      const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(pe.base[pe.rank] + AR_FLAG_BYTES) +
                               ((int64_t)buf * pe.world + src) * pe.slot_elems + r * K + blk * 32;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 raw = ld_volatile_u4(reinterpret_cast<const uint4*>(p) + i);
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[8 * i + k] += __bfloat162float(e[k]);
      }
    }
    // the reduced partial is rounded to bf16 (as a stored GEMM output would be) before the residual add
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __bfloat162float(__float2bfloat16(v[i]));
    if (res_in != nullptr) {
      const __nv_bfloat16* rr = res_in + r * (int64_t)K + blk * 32;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 raw = reinterpret_cast<const uint4*>(rr)[i];
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[8 * i + k] += __bfloat162float(e[k]);
      }
    }
    if (res_out != nullptr) {
      __nv_bfloat16* ro = res_out + r * (int64_t)K + blk * 32;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 raw;
        __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          e[k] = __float2bfloat16(v[8 * i + k]);
          v[8 * i + k] = __bfloat162float(e[k]);
        }
        reinterpret_cast<uint4*>(ro)[i] = raw;
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) sred[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sred[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) sred[0] = t;
  }
  __syncthreads();
  pdl_trigger();
  if (!act) return;
  const float rrs = rsqrtf(sred[0] / (float)K + eps);
  const __nv_bfloat16* wb = w + blk * 32;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 raw = reinterpret_cast<const uint4*>(wb)[i];
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float wv = __bfloat162float(e[k]);
      if (plus_one) wv += 1.f;
      v[8 * i + k] = v[8 * i + k] * rrs * wv;
    }
  }
  if (y != nullptr) {
    __nv_bfloat16* yo = y + r * (int64_t)K + blk * 32;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 raw;
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        e[k] = __float2bfloat16(v[8 * i + k]);
        v[8 * i + k] = __bfloat162float(e[k]);
      }
      reinterpret_cast<uint4*>(yo)[i] = raw;
    }
  }
  if (q != nullptr) {
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) am = fmaxf(am, fabsf(v[i]));
    const int e = mx_exponent(am, 448.f);
    const float si = exp2i(-e);
    uint8_t* qo = q + r * (int64_t)K + blk * 32;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint4 raw;
      uint8_t* b8 = reinterpret_cast<uint8_t*>(&raw);
#pragma unroll
      for (int k = 0; k < 16; ++k) b8[k] = f32_to_e4m3(v[16 * i + k] * si);
      reinterpret_cast<uint4*>(qo)[i] = raw;
    }
    sf[sf_offset(r, blk, kblocks)] = (uint8_t)(e + 127);
  }
}

void ar_rmsnorm(torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call, torch::Tensor step,
                int64_t calls_per_step, int64_t T, c10::optional<torch::Tensor> res_in, c10::optional<torch::Tensor> res_out, torch::Tensor w,
                double eps, bool plus_one, c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> q,
                c10::optional<torch::Tensor> sf, torch::Tensor status, double timeout_s) {
  const int64_t K = w.size(0);
  TORCH_CHECK(K % 128 == 0 && K / 32 <= 1024, "ar_rmsnorm: hidden must be a multiple of 128 and <= 32768");
  TORCH_CHECK(T * K <= slot_elems, "ar_rmsnorm: rows exceed the slot");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(w.device());
  ArPeers pe = make_peers(peers, rank, world, slot_elems, K, step, calls_per_step);
  auto bf = [](const c10::optional<torch::Tensor>& t) -> __nv_bfloat16* {
    return (t.has_value() && t->defined()) ? reinterpret_cast<__nv_bfloat16*>(t->data_ptr()) : nullptr;
  };
  auto u8 = [](const c10::optional<torch::Tensor>& t) -> uint8_t* {
    return (t.has_value() && t->defined()) ? t->data_ptr<uint8_t>() : nullptr;
  };
  const int threads = std::max(32, (int)((K / 32 + 31) / 32 * 32));
  launch_pdl(ar_rmsnorm_kernel, dim3((unsigned)T), dim3(threads), 0, at::cuda::getCurrentCUDAStream(),
      pe, (int)call, bf(res_in), bf(res_out), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (int)K, (float)eps,
      plus_one ? 1 : 0, bf(y), u8(q), u8(sf), status.data_ptr<int>(), (uint64_t)(timeout_s * 1e9));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k

namespace r9k {

// ------------------------------------------------------------------------------------------------
// Pull variant: every rank's row-parallel GEMM writes its bf16 partial into its OWN region, buffer
// k % 2 (a static address per call site, so graphs capture it). The consumer kernel raises this
// rank's ready flag for the call in every peer's region (one release store per peer, after the
// producing grid completed), waits for the peers' flags, then reads the peers' partials over NVLink
// and reduces them in rank order together with the residual add, RMSNorm and quantisation.
// Flag words live at [AR_MAX_WORLD .. 2*AR_MAX_WORLD) x 2 buffers of the flag page (per source).
// ------------------------------------------------------------------------------------------------
R9K_DEVINL uint32_t* ar_ready_flag(uint8_t* base, uint32_t buf, int src) {
  return reinterpret_cast<uint32_t*>(base) + 8192 + buf * AR_MAX_WORLD + src;
}

__global__ void ar_pull_rmsnorm_kernel(ArPeers pe, int call, const __nv_bfloat16* __restrict__ res_in,
                                       __nv_bfloat16* __restrict__ res_out, const __nv_bfloat16* __restrict__ w,
                                       int K, float eps, int plus_one, __nv_bfloat16* __restrict__ y,
                                       uint8_t* __restrict__ q, uint8_t* __restrict__ sf, int* status,
                                       uint64_t timeout_ns) {
  pdl_wait();  // this rank's producer grid has completed
  __shared__ float sred[32];
  __shared__ int s_fail;
  const int64_t r = blockIdx.x;
  const int kblocks = K / 32;
  const int blk = threadIdx.x;
  const uint32_t gcall = ar_global_call(pe, call);
  const uint32_t epoch = gcall + 1u;
  const uint32_t buf = (uint32_t)call & 1u;  // static per call site (calls_per_step is even)
  if (threadIdx.x == 0) {
    s_fail = 0;
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int p = 0; p < pe.world; ++p) st_release_sys(ar_ready_flag(pe.base[p], buf, pe.rank), epoch);
    }
  }
  __syncthreads();
  if (threadIdx.x < pe.world) {
    const uint32_t* fl = ar_ready_flag(pe.base[pe.rank], buf, threadIdx.x);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(fl) < epoch) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        s_fail = 1;
        report_error(status, kErrPeerTimeout, 310, threadIdx.x);
        break;
      }
    }
  }
  __syncthreads();
  pdl_trigger();
  const bool act = blk < kblocks && !s_fail;
  float v[32];
  float ss = 0.f;
  if (act) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
    for (int src = 0; src < pe.world; ++src) {  // fixed rank order: identical sums on every rank
      const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(pe.base[src] + AR_FLAG_BYTES) +
                               (int64_t)buf * pe.slot_elems + r * K + blk * 32;
      uint4 raw[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) raw[i] = ld_volatile_u4(reinterpret_cast<const uint4*>(p) + i);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw[i]);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[8 * i + k] += __bfloat162float(e[k]);
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __bfloat162float(__float2bfloat16(v[i]));
    if (res_in != nullptr) {
      const __nv_bfloat16* rr = res_in + r * (int64_t)K + blk * 32;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 raw = reinterpret_cast<const uint4*>(rr)[i];
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[8 * i + k] += __bfloat162float(e[k]);
      }
    }
    if (res_out != nullptr) {
      __nv_bfloat16* ro = res_out + r * (int64_t)K + blk * 32;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 raw;
        __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          e[k] = __float2bfloat16(v[8 * i + k]);
          v[8 * i + k] = __bfloat162float(e[k]);
        }
        reinterpret_cast<uint4*>(ro)[i] = raw;
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) sred[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sred[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) sred[0] = t;
  }
  __syncthreads();
  if (!act) return;
  const float rrs = rsqrtf(sred[0] / (float)K + eps);
  const __nv_bfloat16* wb = w + blk * 32;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 raw = reinterpret_cast<const uint4*>(wb)[i];
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float wv = __bfloat162float(e[k]);
      if (plus_one) wv += 1.f;
      v[8 * i + k] = v[8 * i + k] * rrs * wv;
    }
  }
  if (y != nullptr) {
    __nv_bfloat16* yo = y + r * (int64_t)K + blk * 32;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 raw;
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        e[k] = __float2bfloat16(v[8 * i + k]);
        v[8 * i + k] = __bfloat162float(e[k]);
      }
      reinterpret_cast<uint4*>(yo)[i] = raw;
    }
  }
  if (q != nullptr) {
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) am = fmaxf(am, fabsf(v[i]));
    const int e = mx_exponent(am, 448.f);
    const float si = exp2i(-e);
    uint8_t* qo = q + r * (int64_t)K + blk * 32;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint4 raw;
      uint8_t* b8 = reinterpret_cast<uint8_t*>(&raw);
#pragma unroll
      for (int k = 0; k < 16; ++k) b8[k] = f32_to_e4m3(v[16 * i + k] * si);
      reinterpret_cast<uint4*>(qo)[i] = raw;
    }
    sf[sf_offset(r, blk, kblocks)] = (uint8_t)(e + 127);
  }
}

void ar_pull_rmsnorm(torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call,
                     torch::Tensor step, int64_t calls_per_step, int64_t T, c10::optional<torch::Tensor> res_in,
                     c10::optional<torch::Tensor> res_out, torch::Tensor w, double eps, bool plus_one,
                     c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf,
                     torch::Tensor status, double timeout_s) {
  const int64_t K = w.size(0);
  TORCH_CHECK(K % 128 == 0 && K / 32 <= 1024, "ar_pull_rmsnorm: hidden must be a multiple of 128 and <= 32768");
  TORCH_CHECK(T * K <= slot_elems, "ar_pull_rmsnorm: rows exceed the buffer");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(w.device());
  ArPeers pe = make_peers(peers, rank, world, slot_elems, K, step, calls_per_step);
  auto bf = [](const c10::optional<torch::Tensor>& t) -> __nv_bfloat16* {
    return (t.has_value() && t->defined()) ? reinterpret_cast<__nv_bfloat16*>(t->data_ptr()) : nullptr;
  };
  auto u8 = [](const c10::optional<torch::Tensor>& t) -> uint8_t* {
    return (t.has_value() && t->defined()) ? t->data_ptr<uint8_t>() : nullptr;
  };
  const int threads = std::max(32, (int)((K / 32 + 31) / 32 * 32));
  TORCH_CHECK(launch_pdl(ar_pull_rmsnorm_kernel, dim3((unsigned)T), dim3(threads), 0, at::cuda::getCurrentCUDAStream(),
                         pe, (int)call, bf(res_in), bf(res_out), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                         (int)K, (float)eps, plus_one ? 1 : 0, bf(y), u8(q), u8(sf), status.data_ptr<int>(),
                         (uint64_t)(timeout_s * 1e9)) == cudaSuccess,
              "ar_pull_rmsnorm launch");
}

}  // namespace r9k

namespace r9k {

// ------------------------------------------------------------------------------------------------
// LL variant (default): producers store their bf16 partial straight into every rank's LL slot with
// the call's epoch in each 8-byte word (GEMM epilogue, or ll_push for other producers); the consumer
// polls its own region until every word of every source carries the epoch, then reduces in rank
// order. Data and "ready" travel in the same NVLink write, so the consumer sees a source's data one
// one-way NVLink latency after the producer stored it: no fence, no flag round trip, no remote load.
//
// The consumer does not wait on the preceding grid (its inputs announce themselves by epoch) and
// lets the next kernel launch at once. Safe because (a) every producer triggers its dependents only
// after its own griddepcontrol.wait returned, so when the consumer starts every kernel before the
// producer has completed (the residual it reads, the step counter); (b) buffer k % 2 is rewritten
// at call k + 2 only after every rank passed call k + 1, whose data each rank produced after its call
// k consumer finished (the argument of the pull variant).
// ------------------------------------------------------------------------------------------------
__global__ void ll_push_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, ArPeers pe, int H, int call) {
  pdl_wait();
  pdl_trigger();
  const uint32_t epoch = ar_global_call(pe, call) + 1u;
  const uint32_t buf = (uint32_t)call & 1u;
  const int t = blockIdx.y;
  const int e0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (e0 >= H) return;
  const uint4 v = *reinterpret_cast<const uint4*>(x + (int64_t)t * ldx + e0);
#pragma unroll
  for (int p = 0; p < AR_MAX_WORLD; ++p) {
    if (p >= pe.world) break;
    uint32_t* d = ar_ll_slot(pe, p, buf, pe.rank) + (int64_t)t * H + e0;
    st_ll16(d, v.x, v.y, epoch);
    st_ll16(d + 4, v.z, v.w, epoch);
  }
}

void ll_push(torch::Tensor x, torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call,
             torch::Tensor step, int64_t calls_per_step) {
  const int64_t T = x.size(0), H = x.size(1);
  TORCH_CHECK(x.dtype() == torch::kBFloat16 && x.stride(1) == 1 && x.stride(0) % 8 == 0, "ll_push: bf16 rows");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0, "ll_push: 16-byte aligned rows");
  TORCH_CHECK(H % 256 == 0 && T * H <= slot_elems, "ll_push: H % 256 and T*H within the slot");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  ArPeers pe = make_peers(peers, rank, world, slot_elems, H, step, calls_per_step);
  const int threads = 128;
  TORCH_CHECK(launch_pdl(ll_push_kernel, dim3((unsigned)((H / 8 + threads - 1) / threads), (unsigned)T), dim3(threads),
                         0, at::cuda::getCurrentCUDAStream(), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                         x.stride(0), pe, (int)H, (int)call) == cudaSuccess,
              "ll_push launch");
}

// Consumer: one CTA per token row, K / 8 threads, thread i owns elements [8 i, 8 i + 8) -- two 16-byte
// LL words per source, all W x 2 loads in flight together (W is a template parameter).
template <int W>
__global__ void __launch_bounds__(1024) ar_ll_rmsnorm_kernel(
    ArPeers pe, int call, const __nv_bfloat16* __restrict__ res_in, __nv_bfloat16* __restrict__ res_out,
    const __nv_bfloat16* __restrict__ w, int K, float eps, int plus_one, __nv_bfloat16* __restrict__ y,
    uint8_t* __restrict__ q, uint8_t* __restrict__ sf, int* status, uint64_t timeout_ns) {
  pdl_trigger();  // the next GEMM may launch and stream its weights (it waits for this grid's results)
  __shared__ float sred[32];
  __shared__ int s_fail;
  const int r = blockIdx.x;
  const int tid = threadIdx.x;
  const int e0 = tid * 8;
  const uint32_t epoch = ar_global_call(pe, call) + 1u;
  const uint32_t buf = (uint32_t)call & 1u;
  if (tid == 0) s_fail = 0;
  __syncthreads();
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = 0.f;
  uint4 raw[W][2];
  const uint32_t* src[W];
#pragma unroll
  for (int s = 0; s < W; ++s) src[s] = ar_ll_slot(pe, pe.rank, buf, s) + (int64_t)r * K + e0;
  uint32_t pending = (1u << (2 * W)) - 1u;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll
    for (int s = 0; s < W; ++s)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t bit = 1u << (2 * s + h);
        if (pending & bit) {
          raw[s][h] = ld_ll16(src[s] + 4 * h);
          if (raw[s][h].y == epoch && raw[s][h].w == epoch) pending &= ~bit;
        }
      }
    if (pending == 0u) break;
    if (globaltimer_ns() - t0 > timeout_ns) {
      report_error(status, kErrPeerTimeout, 320, r * 65536 + __ffs(pending) - 1);
      s_fail = 1;
      break;
    }
  }
  __syncthreads();
  if (s_fail) return;  // uniform: no barrier follows for a failed block, and nothing is written
#pragma unroll
  for (int s = 0; s < W; ++s)  // fixed rank order: identical sums on every rank
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw[s][h].x);
      const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw[s][h].z);
      v[4 * h + 0] += __low2float(a);
      v[4 * h + 1] += __high2float(a);
      v[4 * h + 2] += __low2float(b);
      v[4 * h + 3] += __high2float(b);
    }
  // the reduced partial is rounded to bf16 (as a stored GEMM output would be) before the residual add
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(__float2bfloat16(v[i]));
  if (res_in != nullptr) {
    const uint4 rr = *reinterpret_cast<const uint4*>(res_in + (int64_t)r * K + e0);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&rr);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] += __bfloat162float(e[i]);
  }
  {
    uint4 ro;
    __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&ro);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      e[i] = __float2bfloat16(v[i]);
      v[i] = __bfloat162float(e[i]);
    }
    if (res_out != nullptr) *reinterpret_cast<uint4*>(res_out + (int64_t)r * K + e0) = ro;
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) sred[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float t = tid < (int)(blockDim.x >> 5) ? sred[tid] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (tid == 0) sred[0] = t;
  }
  __syncthreads();
  const float rrs = rsqrtf(sred[0] / (float)K + eps);
  {
    const uint4 wr = *reinterpret_cast<const uint4*>(w + e0);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&wr);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float wv = __bfloat162float(e[i]);
      if (plus_one) wv += 1.f;
      v[i] = v[i] * rrs * wv;
    }
  }
  if (y != nullptr) {
    uint4 yo;
    __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&yo);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      e[i] = __float2bfloat16(v[i]);
      v[i] = __bfloat162float(e[i]);
    }
    *reinterpret_cast<uint4*>(y + (int64_t)r * K + e0) = yo;
  }
  if (q != nullptr) {
    // MX block of 32 elements = 4 consecutive threads
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    const int ex = mx_exponent(am, 448.f);
    const float si = exp2i(-ex);
    uint2 qo;
    uint8_t* b8 = reinterpret_cast<uint8_t*>(&qo);
#pragma unroll
    for (int i = 0; i < 8; ++i) b8[i] = f32_to_e4m3(v[i] * si);
    *reinterpret_cast<uint2*>(q + (int64_t)r * K + e0) = qo;
    if ((tid & 3) == 0) sf[sf_offset(r, e0 >> 5, K / 32)] = (uint8_t)(ex + 127);
  }
}

void ar_ll_rmsnorm(torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call,
                   torch::Tensor step, int64_t calls_per_step, int64_t T, c10::optional<torch::Tensor> res_in,
                   c10::optional<torch::Tensor> res_out, torch::Tensor w, double eps, bool plus_one,
                   c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf,
                   torch::Tensor status, double timeout_s) {
  const int64_t K = w.size(0);
  TORCH_CHECK(K % 256 == 0 && K / 8 <= 1024, "ar_ll_rmsnorm: hidden must be a multiple of 256 and <= 8192");
  TORCH_CHECK(T * K <= slot_elems, "ar_ll_rmsnorm: rows exceed the slot");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(w.device());
  ArPeers pe = make_peers(peers, rank, world, slot_elems, K, step, calls_per_step);
  auto bf = [](const c10::optional<torch::Tensor>& t) -> __nv_bfloat16* {
    return (t.has_value() && t->defined()) ? reinterpret_cast<__nv_bfloat16*>(t->data_ptr()) : nullptr;
  };
  auto u8 = [](const c10::optional<torch::Tensor>& t) -> uint8_t* {
    return (t.has_value() && t->defined()) ? t->data_ptr<uint8_t>() : nullptr;
  };
  const dim3 grid((unsigned)T), block((unsigned)(K / 8));
  const auto st = at::cuda::getCurrentCUDAStream();
  const uint64_t tmo = (uint64_t)(timeout_s * 1e9);
  const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  cudaError_t e = cudaErrorInvalidValue;
#define R9K_LL(WS)                                                                                                    \
  case WS:                                                                                                            \
    e = launch_pdl(ar_ll_rmsnorm_kernel<WS>, grid, block, 0, st, pe, (int)call, bf(res_in), bf(res_out), wp, (int)K,  \
                   (float)eps, plus_one ? 1 : 0, bf(y), u8(q), u8(sf), status.data_ptr<int>(), tmo);                  \
    break;
  switch (world) {
    R9K_LL(1)
    R9K_LL(2)
    R9K_LL(3)
    R9K_LL(4)
    R9K_LL(5)
    R9K_LL(6)
    R9K_LL(7)
    R9K_LL(8)
    default: break;
  }
#undef R9K_LL
  TORCH_CHECK(e == cudaSuccess, "ar_ll_rmsnorm launch: ", cudaGetErrorString(e));
}

}  // namespace r9k
