// Manifold hyper-connections (mHC) seam for DeepSeek-V4-class models: the post step of the previous
// sublayer folded into the pre step of the next, in two launches per seam.
//
// Residual stream R: [T, 4, H] bf16 (4 parallel residual streams). Per token:
//   post (previous sublayer):  R'[j, h] = bf16( sum_i comb[i, j] R[i, h] + post[j] so[h] )   (no so: R' = R)
//   pre  (next sublayer):      x = R' flattened (k = i H + h), K = 4H
//                              mixes[m] = (x . fn[m]) * rsqrt(sum(x^2) / K + rms_eps),  m < 24
//                              pre  = sigmoid(mixes[0:4]  * scale0 + base[0:4])  + pre_eps
//                              post = sigmoid(mixes[4:8]  * scale1 + base[4:8])  * post_mult
//                              comb = sinkhorn(softmax_j(mixes[8:24] * scale2 + base[8:24]) + eps)
//                              li[h] = bf16( sum_i pre[i] R'[i, h] )      (the sublayer's input)
// (semantics of vLLM's torch reference model_executor/kernels/mhc/torch.py; the reference's one-launch
// RDNA4 version: kernels/r9k_mhc.hip:144-303.)
//
// Launch 1 (partial): grid (H / 64 chunks, ceil(T / TG)), 256 threads: thread (i = tid / 64, h) forms
// R'[i, h0 + h] for each token of its group, stores it, and multiplies it into the 24 mixes and the
// sum of squares; a block reduction writes 25 partials per (token, chunk). The chunk's fn slice
// (24 x 256 fp32) is loaded once per CTA and reused by every token of the group.
// Launch 2 (finish): grid (H / 128, T), 128 threads: every CTA reduces its token's partials in chunk
// order (identical in every CTA, so the gates agree bit for bit), computes the gates and the Sinkhorn
// normalisation, and writes li for its 128 h; CTA 0 also writes the token's post and comb.
// Every sum runs in a fixed order: results do not depend on the batch or on scheduling.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

namespace {
constexpr int HC = 4, NMIX = 24, NP = NMIX + 1, CHK = 64, TG = 8;

R9K_DEVINL float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
}  // namespace

__global__ void __launch_bounds__(256) mhc_partial_kernel(
    const __nv_bfloat16* __restrict__ R, const __nv_bfloat16* __restrict__ so, const float* __restrict__ post_in,
    const float* __restrict__ comb_in, const float* __restrict__ fn, __nv_bfloat16* __restrict__ R_out,
    float* __restrict__ part, int T, int H) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sfn[NMIX][HC * CHK];
  __shared__ float red[8][NP];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int i = tid / CHK, hh = tid % CHK;
  const int h0 = blockIdx.x * CHK, nchunk = gridDim.x;
  const int64_t K = (int64_t)HC * H;
  for (int e = tid; e < NMIX * HC * CHK; e += 256) {
    const int m = e / (HC * CHK), r = e % (HC * CHK);
    sfn[m][r] = fn[(int64_t)m * K + (int64_t)(r / CHK) * H + h0 + (r % CHK)];
  }
  __syncthreads();
  const int t_end = min(T, (int)(blockIdx.y + 1) * TG);
  for (int t = blockIdx.y * TG; t < t_end; ++t) {
    const __nv_bfloat16* Rt = R + (int64_t)t * HC * H;
    float v;
    if (so != nullptr) {
      // fma chain over the source streams in order, then the post term
      float acc = 0.f;
#pragma unroll
      for (int s = 0; s < HC; ++s) acc = fmaf(comb_in[(int64_t)t * HC * HC + s * HC + i], __bfloat162float(Rt[(int64_t)s * H + h0 + hh]), acc);
      acc += post_in[(int64_t)t * HC + i] * __bfloat162float(so[(int64_t)t * H + h0 + hh]);
      const __nv_bfloat16 b = __float2bfloat16(acc);
      v = __bfloat162float(b);
      __syncthreads();  // R_out may alias R: every thread has read its four source streams
      R_out[(int64_t)t * HC * H + (int64_t)i * H + h0 + hh] = b;
    } else {
      v = __bfloat162float(Rt[(int64_t)i * H + h0 + hh]);
      if (R_out != R) R_out[(int64_t)t * HC * H + (int64_t)i * H + h0 + hh] = Rt[(int64_t)i * H + h0 + hh];
    }
    float acc[NP];
#pragma unroll
    for (int m = 0; m < NMIX; ++m) acc[m] = v * sfn[m][tid];
    acc[NMIX] = v * v;
#pragma unroll
    for (int m = 0; m < NP; ++m) {
      float x = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      acc[m] = x;
    }
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < NP; ++m) red[warp][m] = acc[m];
    }
    __syncthreads();
    if (tid < NP) {
      float x = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) x += red[w][tid];
      part[((int64_t)t * nchunk + blockIdx.x) * NP + tid] = x;
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(128) mhc_finish_kernel(
    const __nv_bfloat16* __restrict__ R, const float* __restrict__ part, int nchunk, const float* __restrict__ scale,
    const float* __restrict__ base, float rms_eps, float pre_eps, float sk_eps, float post_mult, int sk_repeat,
    float* __restrict__ post_out, float* __restrict__ comb_out, __nv_bfloat16* __restrict__ li, int H) {
  pdl_wait();
  pdl_trigger();
  __shared__ float mix[NP];
  __shared__ float pre[HC];
  const int t = blockIdx.y, tid = threadIdx.x;
  if (tid < NP) {
    float x = 0.f;
    for (int c = 0; c < nchunk; ++c) x += part[((int64_t)t * nchunk + c) * NP + tid];
    mix[tid] = x;
  }
  __syncthreads();
  if (tid == 0) {
    const float r = rsqrtf(mix[NMIX] / (float)(HC * H) + rms_eps);
    float m[NMIX];
#pragma unroll
    for (int k = 0; k < NMIX; ++k) m[k] = mix[k] * r;
    float pst[HC], c[HC][HC];
#pragma unroll
    for (int k = 0; k < HC; ++k) {
      pre[k] = sigmoidf_(m[k] * scale[0] + base[k]) + pre_eps;
      pst[k] = sigmoidf_(m[HC + k] * scale[1] + base[HC + k]) * post_mult;
    }
#pragma unroll
    for (int a = 0; a < HC; ++a) {
      float mx = -INFINITY;
#pragma unroll
      for (int b = 0; b < HC; ++b) {
        c[a][b] = m[2 * HC + a * HC + b] * scale[2] + base[2 * HC + a * HC + b];
        mx = fmaxf(mx, c[a][b]);
      }
      float s = 0.f;
#pragma unroll
      for (int b = 0; b < HC; ++b) {
        c[a][b] = expf(c[a][b] - mx);
        s += c[a][b];
      }
#pragma unroll
      for (int b = 0; b < HC; ++b) c[a][b] = c[a][b] / s + sk_eps;
    }
    // column pass, then (repeat - 1) x (row pass, column pass)
    for (int it = 0; it < sk_repeat; ++it) {
      if (it > 0) {
#pragma unroll
        for (int a = 0; a < HC; ++a) {
          float s = 0.f;
#pragma unroll
          for (int b = 0; b < HC; ++b) s += c[a][b];
#pragma unroll
          for (int b = 0; b < HC; ++b) c[a][b] = c[a][b] / (s + sk_eps);
        }
      }
#pragma unroll
      for (int b = 0; b < HC; ++b) {
        float s = 0.f;
#pragma unroll
        for (int a = 0; a < HC; ++a) s += c[a][b];
#pragma unroll
        for (int a = 0; a < HC; ++a) c[a][b] = c[a][b] / (s + sk_eps);
      }
    }
    if (blockIdx.x == 0) {
#pragma unroll
      for (int k = 0; k < HC; ++k) post_out[(int64_t)t * HC + k] = pst[k];
#pragma unroll
      for (int a = 0; a < HC; ++a)
#pragma unroll
        for (int b = 0; b < HC; ++b) comb_out[(int64_t)t * HC * HC + a * HC + b] = c[a][b];
    }
  }
  __syncthreads();
  const int h = blockIdx.x * 128 + tid;
  if (h < H) {
    const __nv_bfloat16* Rt = R + (int64_t)t * HC * H;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < HC; ++i) acc += pre[i] * __bfloat162float(Rt[(int64_t)i * H + h]);
    li[(int64_t)t * H + h] = __float2bfloat16(acc);
  }
}

// R: [T, 4, H] bf16 (read); so/post_in/comb_in: the previous sublayer's output and mixes (or None);
// R_out: [T, 4, H] bf16 (may alias R when so is None); part: fp32 scratch [T, H / 64, 25].
void mhc_seam(torch::Tensor R, c10::optional<torch::Tensor> so, c10::optional<torch::Tensor> post_in,
              c10::optional<torch::Tensor> comb_in, torch::Tensor fn, torch::Tensor scale, torch::Tensor base,
              double rms_eps, double pre_eps, double sk_eps, double post_mult, int64_t sk_repeat, torch::Tensor R_out,
              torch::Tensor post_out, torch::Tensor comb_out, torch::Tensor li, torch::Tensor part) {
  const int64_t T = R.size(0), H = R.size(2);
  if (T == 0) return;
  TORCH_CHECK(R.size(1) == HC && R.is_contiguous() && R_out.is_contiguous() && H % 128 == 0, "mhc_seam: R [T, 4, H], H % 128");
  TORCH_CHECK(fn.dtype() == torch::kFloat32 && fn.size(0) == NMIX && fn.size(1) == HC * H && fn.is_contiguous(), "mhc_seam: fn [24, 4H] f32");
  const int nchunk = (int)(H / CHK);
  TORCH_CHECK(part.numel() >= T * nchunk * NP, "mhc_seam: partial scratch too small");
  const bool has_so = so.has_value() && so->defined();
  if (has_so) TORCH_CHECK(post_in.has_value() && comb_in.has_value(), "mhc_seam: so needs post and comb mixes");
  const at::cuda::CUDAGuard guard(R.device());
  auto st = at::cuda::getCurrentCUDAStream();
  auto bf = [](const torch::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); };
  launch_pdl(mhc_partial_kernel, dim3(nchunk, (unsigned)((T + TG - 1) / TG)), dim3(256), 0, st, bf(R),
             has_so ? bf(*so) : nullptr, has_so ? post_in->data_ptr<float>() : nullptr,
             has_so ? comb_in->data_ptr<float>() : nullptr, fn.data_ptr<float>(),
             reinterpret_cast<__nv_bfloat16*>(R_out.data_ptr()), part.data_ptr<float>(), (int)T, (int)H);
  launch_pdl(mhc_finish_kernel, dim3((unsigned)((H + 127) / 128), (unsigned)T), dim3(128), 0, st, bf(R_out),
             part.data_ptr<float>(), nchunk, scale.data_ptr<float>(), base.data_ptr<float>(), (float)rms_eps,
             (float)pre_eps, (float)sk_eps, (float)post_mult, (int)sk_repeat, post_out.data_ptr<float>(),
             comb_out.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(li.data_ptr()), (int)H);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k
