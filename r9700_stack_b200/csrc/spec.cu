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
