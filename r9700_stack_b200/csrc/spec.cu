// Speculative decoding glue kernels.
//
//   spec_accept: greedy acceptance of draft tokens on the device. A verify step feeds, per
//   sequence, [last token, d_1 .. d_k] and samples the target's argmax y_0 .. y_k at every position;
//   drafts are accepted while d_{i+1} == y_i, so acc_len = 1 + (number of accepted drafts) tokens
//   enter the recurrent state at commit and y_{acc_len - 1} is the bonus token.
//   (reference: the accept rule vLLM's rejection sampler applies at temperature 0, used by the
//   reference's MTP / DFlash / DSpark paths: r9700_vllm/spec/mtp_rocm.py, models/dflash.py.)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

__global__ void spec_accept_kernel(const int32_t* __restrict__ input_ids, const int64_t* __restrict__ target,
                                   const int32_t* __restrict__ seq_start, const int32_t* __restrict__ seq_len,
                                   int32_t* __restrict__ acc_len, int S) {
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= S) return;
  const int t0 = seq_start[s], n = seq_len[s];
  int j = 0;
  while (j < n - 1 && (int64_t)input_ids[t0 + 1 + j] == target[t0 + j]) ++j;
  acc_len[s] = n > 0 ? j + 1 : 0;
}

void spec_accept(torch::Tensor input_ids, torch::Tensor target, torch::Tensor seq_start, torch::Tensor seq_len,
                 torch::Tensor acc_len) {
  const int64_t S = seq_start.size(0);
  if (S == 0) return;
  TORCH_CHECK(target.dtype() == torch::kInt64 && input_ids.dtype() == torch::kInt32, "spec_accept: dtypes");
  const at::cuda::CUDAGuard guard(input_ids.device());
  launch_pdl(spec_accept_kernel, dim3((unsigned)((S + 127) / 128)), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
             input_ids.data_ptr<int32_t>(), target.data_ptr<int64_t>(), seq_start.data_ptr<int32_t>(),
             seq_len.data_ptr<int32_t>(), acc_len.data_ptr<int32_t>(), (int)S);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------------------------
// dspark_markov_step: one left-to-right step j of the DSpark draft refinement, for every proposing
// sequence s at once:
//   logit_v = base[s, j, v] + head[v] . embed[prev_s]          (rank-64 bigram correction, fp32 dot)
//   d_s     = first argmax over v
//   c       = sigmoid(conf_w . [h[s, j], embed[d_s]])
//   run_s  *= c;  the draft keeps step j while every step so far kept (step 0 always) and run_s >= min
// Each CTA scores kMkRpt * 256 vocabulary rows for all sequences (a weight row is loaded once into
// registers and dotted with every sequence's previous-token embedding from shared memory) and
// parks one (max, first index) pair per sequence; the CTA that arrives last on the counter folds the
// pairs (lowest index wins ties, as torch.argmax), evaluates the confidence head and updates the
// per-sequence state, then re-arms the counter for the next step. No CTA waits on another.
// (reference: the markov / markov_last / markov_conf kernels of kernels/r9k_dsv4_glue.hip:500-649 and
// install_markov in r9700_vllm/dsv4_glue.py:812; here one launch per draft step does all three.)
constexpr int kMkRank = 64;
constexpr int kMkRpt = 2;

__device__ __forceinline__ float2 bf2_to_f2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ void argmax_merge(float& best, int& bi, float v, int i) {
  if (v > best || (v == best && i < bi)) {
    best = v;
    bi = i;
  }
}

__global__ void __launch_bounds__(256) dspark_markov_kernel(
    const float* __restrict__ base, int km, int j, int V, const uint16_t* __restrict__ embed,
    const uint16_t* __restrict__ head, const uint16_t* __restrict__ hrows, int H, const uint16_t* __restrict__ conf_w,
    float min_conf, int64_t* __restrict__ prev, float* __restrict__ run, int32_t* __restrict__ lengths,
    int64_t* __restrict__ drafts, float2* __restrict__ part, int* __restrict__ counter, int S) {
  extern __shared__ float e_prev[];  // [S][kMkRank]
  __shared__ float red_v[8];
  __shared__ int red_i[8];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < S * kMkRank; i += 256) {
    const int64_t t = prev[i / kMkRank];
    e_prev[i] = __uint_as_float((uint32_t)embed[t * kMkRank + (i % kMkRank)] << 16);
  }
  // this thread's weight rows, kept in registers across sequences
  uint4 w[kMkRpt][kMkRank / 8];
  int rows[kMkRpt];
#pragma unroll
  for (int r = 0; r < kMkRpt; ++r) {
    rows[r] = (blockIdx.x * kMkRpt + r) * 256 + tid;
    const uint4* src = reinterpret_cast<const uint4*>(head + (int64_t)min(rows[r], V - 1) * kMkRank);
#pragma unroll
    for (int c = 0; c < kMkRank / 8; ++c) w[r][c] = __ldg(src + c);
  }
  __syncthreads();
  for (int s = 0; s < S; ++s) {
    const float* e = e_prev + s * kMkRank;
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int r = 0; r < kMkRpt; ++r) {
      if (rows[r] >= V) continue;
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < kMkRank / 8; ++c) {
        const uint32_t u[4] = {w[r][c].x, w[r][c].y, w[r][c].z, w[r][c].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 f = bf2_to_f2(u[h]);
          acc = fmaf(f.x, e[c * 8 + 2 * h], acc);
          acc = fmaf(f.y, e[c * 8 + 2 * h + 1], acc);
        }
      }
      const float v = base[((int64_t)s * km + j) * V + rows[r]] + acc;
      if (v > best) {  // rows ascend within a thread: the first maximum stays
        best = v;
        bi = rows[r];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_merge(best, bi, ov, oi);
    }
    if (lane == 0) {
      red_v[warp] = best;
      red_i[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      for (int q = 1; q < 8; ++q) argmax_merge(best, bi, red_v[q], red_i[q]);
      part[(int64_t)s * gridDim.x + blockIdx.x] = make_float2(best, __int_as_float(bi));
    }
    __syncthreads();
  }
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(counter, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // last CTA: one warp per sequence folds the parked pairs and runs the confidence head
  for (int s = warp; s < S; s += 8) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int b = lane; b < (int)gridDim.x; b += 32) {
      const float2 pr = __ldcg(part + (int64_t)s * gridDim.x + b);
      argmax_merge(best, bi, pr.x, __float_as_int(pr.y));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_merge(best, bi, ov, oi);
    }
    const int d = (bi >= 0 && bi < V) ? bi : 0;
    const uint16_t* hr = hrows + ((int64_t)s * km + j) * H;
    float z = 0.f;
    for (int i = lane; i < H; i += 32)
      z = fmaf(__uint_as_float((uint32_t)hr[i] << 16), __uint_as_float((uint32_t)conf_w[i] << 16), z);
    for (int i = lane; i < kMkRank; i += 32)
      z = fmaf(__uint_as_float((uint32_t)embed[(int64_t)d * kMkRank + i] << 16),
               __uint_as_float((uint32_t)conf_w[H + i] << 16), z);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    if (lane == 0) {
      const float c = 1.f / (1.f + expf(-z));
      const float r = (j == 0 ? 1.f : run[s]) * c;
      run[s] = r;
      if (j == 0) lengths[s] = 1;
      else if (lengths[s] == j && r >= min_conf) lengths[s] = j + 1;
      drafts[(int64_t)s * km + j] = d;
      prev[s] = d;
    }
  }
  if (tid == 0) *counter = 0;
}

void dspark_markov_step(torch::Tensor base, int64_t j, torch::Tensor embed, torch::Tensor head, torch::Tensor hrows,
                        torch::Tensor conf_w, double min_conf, torch::Tensor prev, torch::Tensor run,
                        torch::Tensor lengths, torch::Tensor drafts, torch::Tensor part, torch::Tensor counter) {
  const int64_t S = base.size(0), km = base.size(1), V = base.size(2);
  if (S == 0) return;
  TORCH_CHECK(base.dtype() == torch::kFloat32 && base.is_contiguous(), "dspark_markov_step: base fp32 [S, k, V]");
  TORCH_CHECK(embed.size(1) == kMkRank && head.size(1) == kMkRank && embed.size(0) >= V && head.size(0) >= V,
              "dspark_markov_step: rank-64 embed / head with a row per vocabulary entry");
  TORCH_CHECK(embed.dtype() == torch::kBFloat16 && head.dtype() == torch::kBFloat16 &&
                  hrows.dtype() == torch::kBFloat16 && conf_w.dtype() == torch::kBFloat16,
              "dspark_markov_step: bf16 weights and rows");
  TORCH_CHECK(embed.is_contiguous() && head.is_contiguous() && hrows.is_contiguous() && conf_w.is_contiguous(),
              "dspark_markov_step: contiguous operands");
  const int64_t H = hrows.size(-1);
  TORCH_CHECK(hrows.numel() >= S * km * H && conf_w.numel() == H + kMkRank, "dspark_markov_step: hidden sizes");
  TORCH_CHECK(j >= 0 && j < km && S <= 64, "dspark_markov_step: step index / at most 64 sequences");
  TORCH_CHECK(prev.dtype() == torch::kInt64 && drafts.dtype() == torch::kInt64 && run.dtype() == torch::kFloat32 &&
                  lengths.dtype() == torch::kInt32 && counter.dtype() == torch::kInt32,
              "dspark_markov_step: state dtypes");
  TORCH_CHECK(drafts.numel() >= S * km && prev.numel() >= S && run.numel() >= S && lengths.numel() >= S,
              "dspark_markov_step: state sizes");
  const int grid = (int)((V + 256 * kMkRpt - 1) / (256 * kMkRpt));
  TORCH_CHECK(part.dtype() == torch::kFloat32 && part.numel() >= 2 * S * grid, "dspark_markov_step: partials");
  const at::cuda::CUDAGuard guard(base.device());
  const size_t smem = (size_t)S * kMkRank * sizeof(float);
  dspark_markov_kernel<<<grid, 256, smem, at::cuda::getCurrentCUDAStream()>>>(
      base.data_ptr<float>(), (int)km, (int)j, (int)V, reinterpret_cast<const uint16_t*>(embed.data_ptr()),
      reinterpret_cast<const uint16_t*>(head.data_ptr()), reinterpret_cast<const uint16_t*>(hrows.data_ptr()), (int)H,
      reinterpret_cast<const uint16_t*>(conf_w.data_ptr()), (float)min_conf, prev.data_ptr<int64_t>(),
      run.data_ptr<float>(), lengths.data_ptr<int32_t>(), drafts.data_ptr<int64_t>(),
      reinterpret_cast<float2*>(part.data_ptr<float>()), counter.data_ptr<int32_t>(), (int)S);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k

namespace r9k {

// Device trace stamp: buf[slot] = %globaltimer (ns). One thread; captured into CUDA graphs like any
// kernel, so replayed steps are traced too. The stamp lands when the preceding work on the stream
// has finished (stream order; PDL is not used here on purpose).
__global__ void trace_stamp_kernel(int64_t* buf, int64_t slot) { buf[slot] = (int64_t)globaltimer_ns(); }

void trace_stamp(torch::Tensor buf, int64_t slot) {
  TORCH_CHECK(buf.dtype() == torch::kInt64 && slot >= 0 && slot < buf.numel(), "trace_stamp: slot out of range");
  const at::cuda::CUDAGuard guard(buf.device());
  trace_stamp_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(buf.data_ptr<int64_t>(), slot);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k
