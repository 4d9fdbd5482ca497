// Hyper-connection glue (Flash-Next / Qwen4Exp class): the residual stream is HC copies of the hidden
// state, X [T, HC * HD]. Around every block two per-token elementwise kernels run:
//
//   gate_mix     y[n, i] = (1 / HC) * sum_s sigmoid(g[n, s*HD + i]) * x[n, s*HD + i]        (i < HD)
//                (the block's input from the normalised streams; g is per token or one shared row)
//   combine_norm per (n, s): inj = 2 * sigmoid(l[n, s] / HC)
//                out[n, s*HD + i] = bf16(res[n, s*HD + i] + block[n, i] * inj)   (stored back into res)
//                y = out * rsqrt(mean_i(out^2) + eps);  y += y * w[s*HD + i]  -> bf16   (normalised stream)
//
// fp32 math, bf16 in and out, the rounding points above. gate_mix: one thread per 8 elements of a row;
// combine_norm: one 128-thread CTA per (row, stream) holding its row slice in registers between the
// two passes (HD <= 8192). (reference: kernels/r9k_hc.hip:4-14 for the two formulas.)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

constexpr int HC_MAX = 8;
constexpr int HC_NT = 128;
constexpr int HC_VMAX = 8;  // 16-byte vectors per thread: HD <= 128 * 8 * 8

R9K_DEVINL float hc_sigmoid(float x) { return 1.f / (1.f + __expf(-x)); }

__global__ void hc_gate_mix_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ g,
                                   int64_t ldg, int HC, int HD, __nv_bfloat16* __restrict__ y, int64_t ldy, int T) {
  pdl_wait();
  pdl_trigger();
  const int n = blockIdx.y;
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (n >= T || i >= HD) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < HC; ++s) {
    const uint4 xv = *reinterpret_cast<const uint4*>(x + (int64_t)n * ldx + (int64_t)s * HD + i);
    const uint4 gv = *reinterpret_cast<const uint4*>(g + (int64_t)n * ldg + (int64_t)s * HD + i);
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
    const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] += hc_sigmoid(__bfloat162float(ge[k])) * __bfloat162float(xe[k]);
  }
  const float inv = 1.f / (float)HC;
  uint4 ov;
  __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
  for (int k = 0; k < 4; ++k) ob[k] = __floats2bfloat162_rn(acc[2 * k] * inv, acc[2 * k + 1] * inv);
  *reinterpret_cast<uint4*>(y + (int64_t)n * ldy + i) = ov;
}

__global__ void __launch_bounds__(HC_NT) hc_combine_norm_kernel(__nv_bfloat16* __restrict__ res, int64_t ldr,
                                                                const __nv_bfloat16* __restrict__ blk, int64_t ldb,
                                                                const float* __restrict__ l, int64_t ldl,
                                                                const __nv_bfloat16* __restrict__ w, int w_per_stream,
                                                                int HC, int HD, float eps,
                                                                __nv_bfloat16* __restrict__ y, int64_t ldy) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[HC_NT / 32];
  const int n = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
  const float inj = blk != nullptr ? 2.f * hc_sigmoid(l[(int64_t)n * ldl + s] / (float)HC) : 0.f;
  __nv_bfloat16* rr = res + (int64_t)n * ldr + (int64_t)s * HD;
  const int nv = HD / 8;
  uint4 keep[HC_VMAX];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < HC_VMAX; ++j) {
    const int v = tid + j * HC_NT;
    if (v < nv) {
      uint4 rv = reinterpret_cast<const uint4*>(rr)[v];
      __nv_bfloat16* re = reinterpret_cast<__nv_bfloat16*>(&rv);
      if (blk != nullptr) {
        const uint4 bv = reinterpret_cast<const uint4*>(blk + (int64_t)n * ldb)[v];
        const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&bv);
#pragma unroll
        for (int k = 0; k < 8; ++k) re[k] = __float2bfloat16(__bfloat162float(re[k]) + __bfloat162float(be[k]) * inj);
        reinterpret_cast<uint4*>(rr)[v] = rv;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float f = __bfloat162float(re[k]);
        ss += f * f;
      }
      keep[j] = rv;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < HC_NT / 32; ++k) tot += red[k];
  const float rrms = rsqrtf(tot / (float)HD + eps);
  const __nv_bfloat16* wr = w + (w_per_stream ? (int64_t)s * HD : 0);
  __nv_bfloat16* yr = y + (int64_t)n * ldy + (int64_t)s * HD;
#pragma unroll
  for (int j = 0; j < HC_VMAX; ++j) {
    const int v = tid + j * HC_NT;
    if (v < nv) {
      const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&keep[j]);
      const uint4 wv = reinterpret_cast<const uint4*>(wr)[v];
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
      uint4 ov;
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float t = __bfloat162float(re[k]) * rrms;
        oe[k] = __float2bfloat16(t + t * __bfloat162float(we[k]));
      }
      reinterpret_cast<uint4*>(yr)[v] = ov;
    }
  }
}

void hc_gate_mix(torch::Tensor x, torch::Tensor g, int64_t HC, torch::Tensor y) {
  const int64_t T = x.size(0);
  if (T == 0) return;
  const int64_t HD = y.size(1);
  TORCH_CHECK(HC >= 1 && HC <= HC_MAX && x.size(1) == HC * HD && HD % 8 == 0, "hc_gate_mix: x [T, HC * HD], HD % 8 == 0");
  TORCH_CHECK(g.size(1) == HC * HD && (g.size(0) == T || g.size(0) == 1), "hc_gate_mix: g [T or 1, HC * HD]");
  TORCH_CHECK(x.dtype() == torch::kBFloat16 && g.dtype() == torch::kBFloat16 && y.dtype() == torch::kBFloat16 &&
                  x.stride(1) == 1 && g.stride(1) == 1 && y.stride(1) == 1 && x.stride(0) % 8 == 0 &&
                  (g.size(0) == 1 || g.stride(0) % 8 == 0) && y.stride(0) % 8 == 0,
              "hc_gate_mix: bf16 rows, 16-byte aligned");
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t ldg = g.size(0) == 1 ? 0 : g.stride(0);
  launch_pdl(hc_gate_mix_kernel, dim3((unsigned)((HD / 8 + 127) / 128), (unsigned)T), dim3(128), 0,
             at::cuda::getCurrentCUDAStream(), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
             reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), ldg, (int)HC, (int)HD,
             reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0), (int)T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void hc_combine_norm(torch::Tensor res, c10::optional<torch::Tensor> block, c10::optional<torch::Tensor> l,
                     torch::Tensor w, int64_t HC, double eps, torch::Tensor y) {
  const int64_t T = res.size(0);
  if (T == 0) return;
  const int64_t HD = res.size(1) / HC;
  TORCH_CHECK(HC >= 1 && HC <= HC_MAX && res.size(1) == HC * HD && HD % 8 == 0 && HD <= HC_NT * 8 * HC_VMAX,
              "hc_combine_norm: res [T, HC * HD], HD % 8 == 0, HD <= 8192");
  TORCH_CHECK(res.dtype() == torch::kBFloat16 && y.dtype() == torch::kBFloat16 && w.dtype() == torch::kBFloat16 &&
                  res.stride(1) == 1 && y.stride(1) == 1 && res.stride(0) % 8 == 0 && y.stride(0) % 8 == 0 &&
                  y.size(1) == HC * HD && w.is_contiguous() && (w.numel() == HD || w.numel() == HC * HD),
              "hc_combine_norm: bf16 rows, 16-byte aligned; w [HD] or [HC * HD]");
  const __nv_bfloat16* bp = nullptr;
  const float* lp = nullptr;
  int64_t ldb = 0, ldl = 0;
  if (block.has_value() && block->defined()) {
    TORCH_CHECK(l.has_value() && l->defined() && l->dtype() == torch::kFloat32 && l->size(1) == HC && l->stride(1) == 1,
                "hc_combine_norm: l [T, HC] fp32");
    TORCH_CHECK(block->dtype() == torch::kBFloat16 && block->size(1) == HD && block->stride(1) == 1 &&
                    block->stride(0) % 8 == 0,
                "hc_combine_norm: block [T, HD] bf16");
    bp = reinterpret_cast<const __nv_bfloat16*>(block->data_ptr());
    ldb = block->stride(0);
    lp = l->data_ptr<float>();
    ldl = l->stride(0);
  }
  const at::cuda::CUDAGuard guard(res.device());
  launch_pdl(hc_combine_norm_kernel, dim3((unsigned)T, (unsigned)HC), dim3(HC_NT), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<__nv_bfloat16*>(res.data_ptr()), res.stride(0), bp, ldb, lp, ldl,
             reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), w.numel() == HC * HD ? 1 : 0, (int)HC, (int)HD,
             (float)eps, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Fused norm point: one 256-thread CTA per row does all of
//   l[s]   = y . wl[s]                                (the injection logits, fp32)
//   res_s  = bf16(res_s + y * 2 sigmoid(l[s] / HC))    (stored back)
//   n_s    = bf16(res_s * rsqrt(mean(res_s^2) + eps) * (1 + w_s))
//   out    = bf16((1 / HC) sum_s sigmoid(g_s) n_s)     (the next block's input)
// in two passes over the row (the second re-reads the residual this CTA just wrote). Thread t owns
// the 8-element chunks t, t + 256, ... of every stream, in both passes.
constexpr int HCF_NT = 256;

__global__ void __launch_bounds__(HCF_NT) hc_point_kernel(__nv_bfloat16* __restrict__ res, int64_t ldr,
                                                          const __nv_bfloat16* __restrict__ y, int64_t ldy,
                                                          const __nv_bfloat16* __restrict__ wl,
                                                          const __nv_bfloat16* __restrict__ w, int w_per_stream,
                                                          const __nv_bfloat16* __restrict__ g, int64_t ldg, int HC,
                                                          int HD, float eps, __nv_bfloat16* __restrict__ out,
                                                          int64_t ldo) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[HCF_NT / 32][HC_MAX];
  __shared__ float s_val[HC_MAX];
  const int n = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nc = HD / 8;
  __nv_bfloat16* rr = res + (int64_t)n * ldr;
  const __nv_bfloat16* yr = y != nullptr ? y + (int64_t)n * ldy : nullptr;
  auto block_sum = [&](float (&v)[HC_MAX]) {
#pragma unroll
    for (int s = 0; s < HC_MAX; ++s) {
      if (s >= HC) break;
      float x = v[s];
#pragma unroll
      for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (lane == 0) red[warp][s] = x;
    }
    __syncthreads();
    if (tid < HC) {
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < HCF_NT / 32; ++k) t += red[k][tid];
      s_val[tid] = t;
    }
    __syncthreads();
  };
  float inj[HC_MAX];
#pragma unroll
  for (int s = 0; s < HC_MAX; ++s) inj[s] = 0.f;
  if (yr != nullptr) {
    float dot[HC_MAX];
#pragma unroll
    for (int s = 0; s < HC_MAX; ++s) dot[s] = 0.f;
    for (int c = tid; c < nc; c += HCF_NT) {
      const uint4 yv = reinterpret_cast<const uint4*>(yr)[c];
      const __nv_bfloat16* ye = reinterpret_cast<const __nv_bfloat16*>(&yv);
#pragma unroll
      for (int s = 0; s < HC_MAX; ++s) {
        if (s >= HC) break;
        const uint4 wv = reinterpret_cast<const uint4*>(wl + (int64_t)s * HD)[c];
        const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
        for (int k = 0; k < 8; ++k) dot[s] += __bfloat162float(ye[k]) * __bfloat162float(we[k]);
      }
    }
    block_sum(dot);
#pragma unroll
    for (int s = 0; s < HC_MAX; ++s)
      if (s < HC) inj[s] = 2.f * hc_sigmoid(s_val[s] / (float)HC);
  }
  // pass 1: residual update + per-stream sum of squares
  float ss[HC_MAX];
#pragma unroll
  for (int s = 0; s < HC_MAX; ++s) ss[s] = 0.f;
  for (int c = tid; c < nc; c += HCF_NT) {
    uint4 yv = make_uint4(0, 0, 0, 0);
    if (yr != nullptr) yv = reinterpret_cast<const uint4*>(yr)[c];
    const __nv_bfloat16* ye = reinterpret_cast<const __nv_bfloat16*>(&yv);
#pragma unroll
    for (int s = 0; s < HC_MAX; ++s) {
      if (s >= HC) break;
      uint4 rv = reinterpret_cast<const uint4*>(rr + (int64_t)s * HD)[c];
      __nv_bfloat16* re = reinterpret_cast<__nv_bfloat16*>(&rv);
      if (yr != nullptr) {
#pragma unroll
        for (int k = 0; k < 8; ++k) re[k] = __float2bfloat16(__bfloat162float(re[k]) + __bfloat162float(ye[k]) * inj[s]);
        reinterpret_cast<uint4*>(rr + (int64_t)s * HD)[c] = rv;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float f = __bfloat162float(re[k]);
        ss[s] += f * f;
      }
    }
  }
  block_sum(ss);
  float rrms[HC_MAX];
#pragma unroll
  for (int s = 0; s < HC_MAX; ++s) rrms[s] = s < HC ? rsqrtf(s_val[s] / (float)HD + eps) : 0.f;
  // pass 2: normalise every stream and mix
  const float inv = 1.f / (float)HC;
  const __nv_bfloat16* gr = g + (int64_t)n * ldg;
  for (int c = tid; c < nc; c += HCF_NT) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < HC_MAX; ++s) {
      if (s >= HC) break;
      const uint4 rv = reinterpret_cast<const uint4*>(rr + (int64_t)s * HD)[c];
      const uint4 wv = reinterpret_cast<const uint4*>(w + (w_per_stream ? (int64_t)s * HD : 0))[c];
      const uint4 gv = reinterpret_cast<const uint4*>(gr + (int64_t)s * HD)[c];
      const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rv);
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
      const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float t = __bfloat162float(re[k]) * rrms[s];
        const float nv = __bfloat162float(__float2bfloat16(t + t * __bfloat162float(we[k])));
        acc[k] += hc_sigmoid(__bfloat162float(ge[k])) * nv;
      }
    }
    uint4 ov;
    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int k = 0; k < 4; ++k) ob[k] = __floats2bfloat162_rn(acc[2 * k] * inv, acc[2 * k + 1] * inv);
    reinterpret_cast<uint4*>(out + (int64_t)n * ldo)[c] = ov;
  }
}

// Register-resident variant for rows of at most R x 256 chunks (used with R = 1, HD <= 2048): every load of the
// point (block output, residual streams, logit weights, norm weights, gates) is issued up front, so the
// point costs one memory round trip plus two block reductions instead of a dependent chain of passes.
constexpr int HCR = 4;  // streams held in registers by the variant below

template <int R>
__global__ void __launch_bounds__(HCF_NT) hc_point_reg_kernel(__nv_bfloat16* __restrict__ res, int64_t ldr,
                                                              const __nv_bfloat16* __restrict__ y, int64_t ldy,
                                                              const __nv_bfloat16* __restrict__ wl,
                                                              const __nv_bfloat16* __restrict__ w, int w_per_stream,
                                                              const __nv_bfloat16* __restrict__ g, int64_t ldg, int HC,
                                                              int HD, float eps, __nv_bfloat16* __restrict__ out,
                                                              int64_t ldo) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[HCF_NT / 32][HC_MAX];
  __shared__ float s_val[HC_MAX];
  const int n = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nc = HD / 8;
  __nv_bfloat16* rr = res + (int64_t)n * ldr;
  const __nv_bfloat16* yr = y != nullptr ? y + (int64_t)n * ldy : nullptr;
  const __nv_bfloat16* gr = g + (int64_t)n * ldg;
  uint4 yv[R], rv[R][HCR], lv[R][HCR], wv[R][HCR], gv[R][HCR];
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int c = tid + j * HCF_NT;
    const bool in = c < nc;
    yv[j] = (in && yr != nullptr) ? reinterpret_cast<const uint4*>(yr)[c] : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int s = 0; s < HCR; ++s) {
      if (s >= HC) break;
      rv[j][s] = in ? reinterpret_cast<const uint4*>(rr + (int64_t)s * HD)[c] : make_uint4(0, 0, 0, 0);
      lv[j][s] = (in && yr != nullptr) ? reinterpret_cast<const uint4*>(wl + (int64_t)s * HD)[c] : make_uint4(0, 0, 0, 0);
      wv[j][s] = in ? reinterpret_cast<const uint4*>(w + (w_per_stream ? (int64_t)s * HD : 0))[c] : make_uint4(0, 0, 0, 0);
      gv[j][s] = in ? reinterpret_cast<const uint4*>(gr + (int64_t)s * HD)[c] : make_uint4(0, 0, 0, 0);
    }
  }
  auto block_sum = [&](float (&v)[HCR]) {
#pragma unroll
    for (int s = 0; s < HCR; ++s) {
      if (s >= HC) break;
      float x = v[s];
#pragma unroll
      for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (lane == 0) red[warp][s] = x;
    }
    __syncthreads();
    if (tid < HC) {
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < HCF_NT / 32; ++k) t += red[k][tid];
      s_val[tid] = t;
    }
    __syncthreads();
  };
  float inj[HCR];
#pragma unroll
  for (int s = 0; s < HCR; ++s) inj[s] = 0.f;
  if (yr != nullptr) {
    float dot[HCR];
#pragma unroll
    for (int s = 0; s < HCR; ++s) dot[s] = 0.f;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const __nv_bfloat16* ye = reinterpret_cast<const __nv_bfloat16*>(&yv[j]);
#pragma unroll
      for (int s = 0; s < HCR; ++s) {
        if (s >= HC) break;
        const __nv_bfloat16* le = reinterpret_cast<const __nv_bfloat16*>(&lv[j][s]);
#pragma unroll
        for (int k = 0; k < 8; ++k) dot[s] += __bfloat162float(ye[k]) * __bfloat162float(le[k]);
      }
    }
    block_sum(dot);
#pragma unroll
    for (int s = 0; s < HCR; ++s)
      if (s < HC) inj[s] = 2.f * hc_sigmoid(s_val[s] / (float)HC);
  }
  float ss[HCR];
#pragma unroll
  for (int s = 0; s < HCR; ++s) ss[s] = 0.f;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int c = tid + j * HCF_NT;
    const __nv_bfloat16* ye = reinterpret_cast<const __nv_bfloat16*>(&yv[j]);
#pragma unroll
    for (int s = 0; s < HCR; ++s) {
      if (s >= HC) break;
      __nv_bfloat16* re = reinterpret_cast<__nv_bfloat16*>(&rv[j][s]);
      if (yr != nullptr) {
#pragma unroll
        for (int k = 0; k < 8; ++k) re[k] = __float2bfloat16(__bfloat162float(re[k]) + __bfloat162float(ye[k]) * inj[s]);
        if (c < nc) reinterpret_cast<uint4*>(rr + (int64_t)s * HD)[c] = rv[j][s];
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float f = __bfloat162float(re[k]);
        ss[s] += f * f;
      }
    }
  }
  block_sum(ss);
  float rrms[HCR];
#pragma unroll
  for (int s = 0; s < HCR; ++s) rrms[s] = s < HC ? rsqrtf(s_val[s] / (float)HD + eps) : 0.f;
  const float inv = 1.f / (float)HC;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int c = tid + j * HCF_NT;
    if (c >= nc) continue;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < HCR; ++s) {
      if (s >= HC) break;
      const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rv[j][s]);
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv[j][s]);
      const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv[j][s]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float t = __bfloat162float(re[k]) * rrms[s];
        const float nv = __bfloat162float(__float2bfloat16(t + t * __bfloat162float(we[k])));
        acc[k] += hc_sigmoid(__bfloat162float(ge[k])) * nv;
      }
    }
    uint4 ov;
    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int k = 0; k < 4; ++k) ob[k] = __floats2bfloat162_rn(acc[2 * k] * inv, acc[2 * k + 1] * inv);
    reinterpret_cast<uint4*>(out + (int64_t)n * ldo)[c] = ov;
  }
}

void hc_point(torch::Tensor res, c10::optional<torch::Tensor> y, torch::Tensor wl, torch::Tensor w, torch::Tensor g,
              int64_t HC, double eps, torch::Tensor out) {
  const int64_t T = res.size(0);
  if (T == 0) return;
  const int64_t HD = out.size(1);
  TORCH_CHECK(HC >= 1 && HC <= HC_MAX && res.size(1) == HC * HD && HD % 8 == 0, "hc_point: res [T, HC * HD], HD % 8 == 0");
  TORCH_CHECK(res.dtype() == torch::kBFloat16 && out.dtype() == torch::kBFloat16 && wl.dtype() == torch::kBFloat16 &&
                  w.dtype() == torch::kBFloat16 && g.dtype() == torch::kBFloat16,
              "hc_point: bf16 tensors");
  TORCH_CHECK(res.stride(1) == 1 && out.stride(1) == 1 && res.stride(0) % 8 == 0 && out.stride(0) % 8 == 0 &&
                  wl.is_contiguous() && wl.size(0) == HC && wl.size(1) == HD && w.is_contiguous() &&
                  (w.numel() == HD || w.numel() == HC * HD) && g.stride(1) == 1 && g.size(1) == HC * HD &&
                  (g.size(0) == 1 || (g.size(0) == T && g.stride(0) % 8 == 0)),
              "hc_point: shapes / 16-byte aligned rows");
  const __nv_bfloat16* yp = nullptr;
  int64_t ldy = 0;
  if (y.has_value() && y->defined()) {
    TORCH_CHECK(y->dtype() == torch::kBFloat16 && y->size(1) == HD && y->stride(1) == 1 && y->stride(0) % 8 == 0,
                "hc_point: y [T, HD] bf16");
    yp = reinterpret_cast<const __nv_bfloat16*>(y->data_ptr());
    ldy = y->stride(0);
  }
  const at::cuda::CUDAGuard guard(res.device());
  const int64_t nc = HD / 8;
  if (HC <= HCR && nc <= HCF_NT) {  // one chunk per thread (HD <= 2048); wider rows spill, so they loop
    launch_pdl(hc_point_reg_kernel<1>, dim3((unsigned)T), dim3(HCF_NT), 0, at::cuda::getCurrentCUDAStream(),
               reinterpret_cast<__nv_bfloat16*>(res.data_ptr()), res.stride(0), yp, ldy,
               reinterpret_cast<const __nv_bfloat16*>(wl.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
               w.numel() == HC * HD ? 1 : 0, reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
               g.size(0) == 1 ? (int64_t)0 : g.stride(0), (int)HC, (int)HD, (float)eps,
               reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  launch_pdl(hc_point_kernel, dim3((unsigned)T), dim3(HCF_NT), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<__nv_bfloat16*>(res.data_ptr()), res.stride(0), yp, ldy,
             reinterpret_cast<const __nv_bfloat16*>(wl.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
             w.numel() == HC * HD ? 1 : 0, reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
             g.size(0) == 1 ? (int64_t)0 : g.stride(0), (int)HC, (int)HD, (float)eps,
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k
