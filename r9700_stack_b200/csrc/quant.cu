// Quantisation and normalisation kernels.
//
//  * rmsnorm_quant: optional residual add, RMSNorm (plain w or Gemma 1+w), bf16 output and/or MXFP8
//    (e4m3 + ue8m0 per 32) output laid out for the GEMM's B operand. This is the producer-side fusion
//    of the reference's per-token fp8 quant (kernels/r9k_moe_mxfp4a8.hip:1683-1780) into the norm.
//  * quant_act_mxfp8: standalone activation quant (kept for R9K_*=stock style A/B and odd producers).
//  * weight quantisers: MXFP4 with an MSE search over exponent shifts -2..+2 (generalising the
//    reference's two-candidate search, r9700_vllm/quant/nvfp4.py:54-76), MXFP8, NVFP4, and the
//    NVFP4 -> MXFP4 load-time conversion (r9700_vllm/quant/nvfp4.py:78-112).
//  * dequantisers used by tests and by fallbacks that need bf16 weights.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

// e2m1 magnitude code for |v| (v already divided by the block scale), round-to-nearest-even,
// saturating at 6.
R9K_DEVINL uint32_t e2m1_code_abs(float v) {
  return (uint32_t)(v > 0.25f) + (uint32_t)(v >= 0.75f) + (uint32_t)(v > 1.25f) + (uint32_t)(v >= 1.75f) +
         (uint32_t)(v > 2.5f) + (uint32_t)(v >= 3.5f) + (uint32_t)(v > 5.0f);
}
R9K_DEVINL float e2m1_value(uint32_t code) {
  const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float m = mag[code & 7];
  return (code & 8) ? -m : m;
}
R9K_DEVINL uint32_t e2m1_encode(float v) {
  const uint32_t c = e2m1_code_abs(fabsf(v));
  return (v < 0.f && c != 0) ? (c | 8u) : c;
}

// ------------------------------------------------------------------------------------------------
// RMSNorm (+ residual) (+ MXFP8 quant)
// ------------------------------------------------------------------------------------------------
// One CTA per row; one thread per 32-element block (the MX quantisation block), so the quantisation
// needs no cross-thread reduction and every load/store is a 16-byte vector.
template <typename TIn>
__global__ void rmsnorm_quant_kernel(const TIn* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ res_in,
                                     __nv_bfloat16* __restrict__ res_out, const __nv_bfloat16* __restrict__ w,
                                     int K, float eps, int plus_one, __nv_bfloat16* __restrict__ y, int64_t ldy,
                                     uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  __shared__ float sred[32];
  const int64_t r = blockIdx.x;
  const int kblocks = K / 32;
  const int blk = threadIdx.x;
  const bool act = blk < kblocks;
  // the norm weights are parameters, not the preceding grid's output: read them before waiting on it
  uint4 wraw[4];
  if (act) {
#pragma unroll
    for (int i = 0; i < 4; ++i) wraw[i] = reinterpret_cast<const uint4*>(w + blk * 32)[i];
  }
  pdl_wait();
  pdl_trigger();  // the next GEMM may start streaming its weights
  float v[32];
  float ss = 0.f;
  if (act) {
    const TIn* xr = x + r * ldx + blk * 32;
    if constexpr (std::is_same<TIn, float>::value) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 f = reinterpret_cast<const float4*>(xr)[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 raw = reinterpret_cast<const uint4*>(xr)[i];
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[8 * i + k] = __bfloat162float(e[k]);
      }
    }
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
          v[8 * i + k] = __bfloat162float(e[k]);  // the residual stream is bf16: normalise what is stored
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
  const float rr = rsqrtf(sred[0] / (float)K + eps);
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&wraw[i]);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float wv = __bfloat162float(e[k]);
      if (plus_one) wv += 1.f;
      v[8 * i + k] = v[8 * i + k] * rr * wv;
    }
  }
  if (y != nullptr) {
    __nv_bfloat16* yo = y + r * ldy + blk * 32;
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

// x: [M, K] bf16 or f32; residual (optional, bf16 [M,K]) is added first and the sum written to
// res_out; then y = rmsnorm(.) * (w or 1+w). Outputs: y (bf16, optional), q/sf (MXFP8, optional).
void rmsnorm_quant(torch::Tensor x, c10::optional<torch::Tensor> res_in, c10::optional<torch::Tensor> res_out,
                   torch::Tensor w, double eps, bool plus_one, c10::optional<torch::Tensor> y,
                   c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf) {
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 32 == 0 && x.stride(1) == 1, "rmsnorm_quant: K % 32 == 0, contiguous rows");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int threads = std::max(32, (int)((K / 32 + 31) / 32 * 32));
  TORCH_CHECK(threads <= 1024, "rmsnorm_quant: K <= 32768");
  TORCH_CHECK((x.stride(0) * x.element_size()) % 16 == 0 && (y.has_value() && y->defined() ? y->stride(0) % 8 == 0 : true),
              "rmsnorm_quant: rows must be 16-byte aligned");
  const size_t smem = 0;
  auto ptr_bf = [](const c10::optional<torch::Tensor>& t) -> __nv_bfloat16* {
    return (t.has_value() && t->defined()) ? reinterpret_cast<__nv_bfloat16*>(t->data_ptr()) : nullptr;
  };
  auto ptr_u8 = [](const c10::optional<torch::Tensor>& t) -> uint8_t* {
    return (t.has_value() && t->defined()) ? t->data_ptr<uint8_t>() : nullptr;
  };
  const int64_t ldy = (y.has_value() && y->defined()) ? y->stride(0) : K;
  if (q.has_value() && q->defined()) {
    TORCH_CHECK(sf.has_value() && sf->defined(), "rmsnorm_quant: q needs sf");
    TORCH_CHECK(sf->numel() >= ((M + 127) / 128) * ((K / 32 + 3) / 4) * 512, "rmsnorm_quant: sf too small");
  }
  if (x.dtype() == torch::kFloat32) {
    launch_pdl(rmsnorm_quant_kernel<float>, dim3((unsigned)M), dim3(threads), smem, st,x.data_ptr<float>(), x.stride(0), ptr_bf(res_in), ptr_bf(res_out),
                                                           reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (int)K,
                                                           (float)eps, plus_one, ptr_bf(y), ldy, ptr_u8(q), ptr_u8(sf));
  } else {
    launch_pdl(rmsnorm_quant_kernel<__nv_bfloat16>, dim3((unsigned)M), dim3(threads), smem, st,
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), ptr_bf(res_in), ptr_bf(res_out),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (int)K, (float)eps, plus_one, ptr_bf(y), ldy, ptr_u8(q),
        ptr_u8(sf));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------------------
// standalone activation quant: bf16 [M, K] (row stride ldx) -> e4m3 [M, K] + ue8m0 chunk scales
// ------------------------------------------------------------------------------------------------
__global__ void quant_act_mxfp8_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int M, int K,
                                       uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  const int kblocks = K / 32;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)M * kblocks;
  for (int64_t b = gw; b < total; b += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t r = b / kblocks;
    const int blk = (int)(b % kblocks);
    const float v = __bfloat162float(x[r * ldx + blk * 32 + lane]);
    float am = fabsf(v);
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const int e = mx_exponent(am, 448.f);
    q[r * K + blk * 32 + lane] = f32_to_e4m3(v * exp2i(-e));
    if (lane == 0) sf[sf_offset(r, blk, kblocks)] = (uint8_t)(e + 127);
  }
}

// ------------------------------------------------------------------------------------------------
// SwiGLU + MXFP8: h = silu(g) * u from the bf16 outputs of the gate and up GEMMs (prefill-sized M,
// where two wide GEMMs beat the dual-accumulator kernel whose per-token quantising epilogue leaves the
// tensor cores idle). Thread = 8 consecutive elements; 4 threads = one 32-element MX block.
// ------------------------------------------------------------------------------------------------
__global__ void swiglu_quant_mxfp8_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ u,
                                          int64_t ld, int M, int N, uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  pdl_wait();
  pdl_trigger();
  const int groups = N / 8;
  const int64_t total = (int64_t)M * groups;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / groups;
    const int c = (int)(i % groups) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(g + r * ld + c);
    const uint4 uv = *reinterpret_cast<const uint4*>(u + r * ld + c);
    const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gv);
    const __nv_bfloat162* uh = reinterpret_cast<const __nv_bfloat162*>(&uv);
    float h[8];
    float am = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = __bfloat1622float2(gh[j]), b = __bfloat1622float2(uh[j]);
      h[2 * j] = silu_f(a.x) * b.x;
      h[2 * j + 1] = silu_f(a.y) * b.y;
      am = fmaxf(am, fmaxf(fabsf(h[2 * j]), fabsf(h[2 * j + 1])));
    }
    // the 4 threads of a block are consecutive lanes (N % 32 == 0, groups of 8 elements)
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    const int e = mx_exponent(am, 448.f);
    const float sc = exp2i(-e);
    uint2 out;
    uint8_t* ob = reinterpret_cast<uint8_t*>(&out);
#pragma unroll
    for (int j = 0; j < 8; ++j) ob[j] = f32_to_e4m3(h[j] * sc);
    *reinterpret_cast<uint2*>(q + r * N + c) = out;
    if ((c & 31) == 0) sf[sf_offset(r, c >> 5, N / 32)] = (uint8_t)(e + 127);
  }
}

void swiglu_quant_mxfp8(torch::Tensor g, torch::Tensor u, torch::Tensor q, torch::Tensor sf) {
  const int64_t M = g.size(0), N = g.size(1);
  TORCH_CHECK(g.dtype() == torch::kBFloat16 && u.dtype() == torch::kBFloat16 && g.sizes() == u.sizes() &&
                  g.stride(0) == u.stride(0) && g.stride(1) == 1 && u.stride(1) == 1 && g.stride(0) % 8 == 0,
              "swiglu_quant_mxfp8: bf16 [M, N] gate / up with one 16-byte-aligned row stride");
  TORCH_CHECK(N % 32 == 0 && q.size(0) >= M && q.size(1) == N, "swiglu_quant_mxfp8: N % 32, q [M, N]");
  TORCH_CHECK(sf.numel() >= ((M + 127) / 128) * ((N / 32 + 3) / 4) * 512, "swiglu_quant_mxfp8: sf too small");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(g.device());
  const int64_t threads = M * (N / 8);
  const int64_t blocks = std::min<int64_t>((threads + 255) / 256, (int64_t)device_sm_count() * 16);
  TORCH_CHECK(launch_pdl(swiglu_quant_mxfp8_kernel, dim3((unsigned)blocks), dim3(256), 0,
                         at::cuda::getCurrentCUDAStream(), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
                         reinterpret_cast<const __nv_bfloat16*>(u.data_ptr()), g.stride(0), (int)M, (int)N,
                         q.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>()) == cudaSuccess,
              "swiglu_quant_mxfp8 launch");
}

void quant_act_mxfp8(torch::Tensor x, torch::Tensor q, torch::Tensor sf) {
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 32 == 0 && x.stride(1) == 1 && x.dtype() == torch::kBFloat16, "quant_act_mxfp8: bf16 [M, K%32]");
  TORCH_CHECK(sf.numel() >= ((M + 127) / 128) * ((K / 32 + 3) / 4) * 512, "quant_act_mxfp8: sf too small");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t warps = M * (K / 32);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((warps * 32 + threads - 1) / threads, 148 * 16);
  launch_pdl(quant_act_mxfp8_kernel, dim3((unsigned)blocks), dim3(threads), 0, at::cuda::getCurrentCUDAStream(),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), (int)M, (int)K, q.data_ptr<uint8_t>(),
      sf.data_ptr<uint8_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------------------
// weight quantisers (one warp per 32-element block)
// ------------------------------------------------------------------------------------------------
// MXFP4 with an exponent search over base-2 .. base+2 (base = ceil(log2(amax/6))), keeping the
// candidate with the lowest squared error (ties -> the larger exponent, i.e. fewer clipped values).
__global__ void quant_w_mxfp4_kernel(const float* __restrict__ w, int64_t N, int K, int search,
                                     uint8_t* __restrict__ packed, uint8_t* __restrict__ sf) {
  const int kblocks = K / 32;
  const int lane = threadIdx.x & 31;
  const int64_t total = N * kblocks;
  for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < total;
       b += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t r = b / kblocks;
    const int blk = (int)(b % kblocks);
    const float v = w[r * K + blk * 32 + lane];
    float am = fabsf(v);
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const int base = mx_exponent(am, 6.f);
    int best_e = base;
    if (search) {
      float best_err = 3.4e38f;
      for (int d = 2; d >= -2; --d) {
        const int e = max(-127, min(127, base + d));
        const float s = exp2i(e);
        const float dq = e2m1_value(e2m1_encode(v / s)) * s;
        float err = (dq - v) * (dq - v);
        for (int o = 16; o > 0; o >>= 1) err += __shfl_xor_sync(0xffffffffu, err, o);
        if (err < best_err) { best_err = err; best_e = e; }
      }
    }
    const uint32_t code = e2m1_encode(v / exp2i(best_e));
    const uint32_t other = __shfl_down_sync(0xffffffffu, code, 1);
    if ((lane & 1) == 0) packed[r * (K / 2) + blk * 16 + (lane >> 1)] = (uint8_t)(code | (other << 4));
    if (lane == 0) sf[sf_offset(r, blk, kblocks)] = (uint8_t)(best_e + 127);
  }
}

__global__ void quant_w_mxfp8_kernel(const float* __restrict__ w, int64_t N, int K, uint8_t* __restrict__ q,
                                     uint8_t* __restrict__ sf) {
  const int kblocks = K / 32;
  const int lane = threadIdx.x & 31;
  const int64_t total = N * kblocks;
  for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < total;
       b += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t r = b / kblocks;
    const int blk = (int)(b % kblocks);
    const float v = w[r * K + blk * 32 + lane];
    float am = fabsf(v);
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const int e = mx_exponent(am, 448.f);
    q[r * K + blk * 32 + lane] = f32_to_e4m3(v * exp2i(-e));
    if (lane == 0) sf[sf_offset(r, blk, kblocks)] = (uint8_t)(e + 127);
  }
}

static int grid_for(int64_t warps) {
  return (int)std::min<int64_t>((warps * 32 + 255) / 256, 148 * 32);
}

void quant_weight_mxfp4(torch::Tensor w, torch::Tensor packed, torch::Tensor sf, bool search) {
  TORCH_CHECK(w.dtype() == torch::kFloat32 && w.is_contiguous(), "quant_weight_mxfp4: contiguous f32");
  const int64_t N = w.size(0), K = w.size(1);
  TORCH_CHECK(K % 32 == 0, "K % 32");
  const at::cuda::CUDAGuard guard(w.device());
  quant_w_mxfp4_kernel<<<grid_for(N * (K / 32)), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      w.data_ptr<float>(), N, (int)K, search ? 1 : 0, packed.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void quant_weight_mxfp8(torch::Tensor w, torch::Tensor q, torch::Tensor sf) {
  TORCH_CHECK(w.dtype() == torch::kFloat32 && w.is_contiguous(), "quant_weight_mxfp8: contiguous f32");
  const int64_t N = w.size(0), K = w.size(1);
  TORCH_CHECK(K % 32 == 0, "K % 32");
  const at::cuda::CUDAGuard guard(w.device());
  quant_w_mxfp8_kernel<<<grid_for(N * (K / 32)), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      w.data_ptr<float>(), N, (int)K, q.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------------------
// NVFP4: e2m1 values, e4m3 scale per 16, fp32 global scale g:  w = v * s / g
// ------------------------------------------------------------------------------------------------
// nvfp4 -> dequantised f32 -> MXFP4 (search), fused: one warp per 32-element MX block (two NVFP4 blocks)
__global__ void nvfp4_to_mxfp4_kernel(const uint8_t* __restrict__ packed_in, const uint8_t* __restrict__ s16,
                                      float inv_g, int64_t N, int K, int search, uint8_t* __restrict__ packed_out,
                                      uint8_t* __restrict__ sf) {
  const int kblocks = K / 32;
  const int lane = threadIdx.x & 31;
  const int64_t total = N * kblocks;
  for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < total;
       b += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t r = b / kblocks;
    const int blk = (int)(b % kblocks);
    const int k = blk * 32 + lane;
    const uint8_t byte = packed_in[r * (K / 2) + (k >> 1)];
    const uint32_t code = (k & 1) ? (byte >> 4) : (byte & 15);
    const float s = e4m3_to_f32(s16[r * (K / 16) + (k >> 4)]);
    const float v = e2m1_value(code) * s * inv_g;
    float am = fabsf(v);
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const int base = mx_exponent(am, 6.f);
    int best_e = base;
    if (search) {
      float best_err = 3.4e38f;
      for (int d = 2; d >= -2; --d) {
        const int e = max(-127, min(127, base + d));
        const float sc = exp2i(e);
        const float dq = e2m1_value(e2m1_encode(v / sc)) * sc;
        float err = (dq - v) * (dq - v);
        for (int o = 16; o > 0; o >>= 1) err += __shfl_xor_sync(0xffffffffu, err, o);
        if (err < best_err) { best_err = err; best_e = e; }
      }
    }
    const uint32_t c = e2m1_encode(v / exp2i(best_e));
    const uint32_t other = __shfl_down_sync(0xffffffffu, c, 1);
    if ((lane & 1) == 0) packed_out[r * (K / 2) + blk * 16 + (lane >> 1)] = (uint8_t)(c | (other << 4));
    if (lane == 0) sf[sf_offset(r, blk, kblocks)] = (uint8_t)(best_e + 127);
  }
}

void nvfp4_to_mxfp4(torch::Tensor packed_in, torch::Tensor s16, double global_scale, torch::Tensor packed_out,
                    torch::Tensor sf, bool search) {
  const int64_t N = packed_in.size(0), K = packed_in.size(1) * 2;
  TORCH_CHECK(K % 32 == 0 && s16.size(1) == K / 16, "nvfp4_to_mxfp4: shapes");
  const at::cuda::CUDAGuard guard(packed_in.device());
  nvfp4_to_mxfp4_kernel<<<grid_for(N * (K / 32)), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      packed_in.data_ptr<uint8_t>(), s16.data_ptr<uint8_t>(), (float)(1.0 / global_scale), N, (int)K, search ? 1 : 0,
      packed_out.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// f32 weights -> NVFP4 (per-16 e4m3 scale s = amax/6 * g, rounded to e4m3; v = w * g / s)
__global__ void quant_w_nvfp4_kernel(const float* __restrict__ w, int64_t N, int K, float g,
                                     uint8_t* __restrict__ packed, uint8_t* __restrict__ s16) {
  const int kb = K / 16;
  const int lane = threadIdx.x & 15;  // half-warp per 16-block
  const int64_t total = N * kb;
  for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4; b < total;
       b += ((int64_t)gridDim.x * blockDim.x) >> 4) {
    const int64_t r = b / kb;
    const int blk = (int)(b % kb);
    const float v = w[r * K + blk * 16 + lane];
    float am = fabsf(v);
    for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o, 16));
    const uint8_t sq = f32_to_e4m3(am / 6.f * g);
    const float s = e4m3_to_f32(sq);
    const uint32_t c = (s > 0.f) ? e2m1_encode(v * g / s) : 0u;
    const uint32_t other = __shfl_down_sync(0xffffffffu, c, 1, 16);
    if ((lane & 1) == 0) packed[r * (K / 2) + blk * 8 + (lane >> 1)] = (uint8_t)(c | (other << 4));
    if (lane == 0) s16[r * kb + blk] = sq;
  }
}

void quant_weight_nvfp4(torch::Tensor w, double global_scale, torch::Tensor packed, torch::Tensor s16) {
  TORCH_CHECK(w.dtype() == torch::kFloat32 && w.is_contiguous(), "quant_weight_nvfp4: contiguous f32");
  const int64_t N = w.size(0), K = w.size(1);
  TORCH_CHECK(K % 16 == 0, "K % 16");
  const at::cuda::CUDAGuard guard(w.device());
  const int64_t hw = N * (K / 16);
  const int blocks = (int)std::min<int64_t>((hw * 16 + 255) / 256, 148 * 32);
  quant_w_nvfp4_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      w.data_ptr<float>(), N, (int)K, (float)global_scale, packed.data_ptr<uint8_t>(), s16.data_ptr<uint8_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------------------
// dequantisers (MX chunk layout -> f32), used by tests and bf16 fallbacks
// ------------------------------------------------------------------------------------------------
__global__ void dequant_mx_kernel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sf, int64_t N, int K,
                                  int fp4, float* __restrict__ out) {
  const int64_t total = N * K;
  const int kblocks = K / 32;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K;
    const int k = (int)(i % K);
    float v;
    if (fp4) {
      const uint8_t byte = q[r * (K / 2) + (k >> 1)];
      v = e2m1_value((k & 1) ? (byte >> 4) : (byte & 15));
    } else {
      v = e4m3_to_f32(q[r * K + k]);
    }
    const int e = (int)sf[sf_offset(r, k >> 5, kblocks)] - 127;
    out[i] = v * exp2i(max(-126, e)) * (e < -126 ? 0.5f : 1.f);
  }
}

void dequant_mx(torch::Tensor q, torch::Tensor sf, bool fp4, torch::Tensor out) {
  const int64_t N = out.size(0), K = out.size(1);
  const at::cuda::CUDAGuard guard(q.device());
  const int blocks = (int)std::min<int64_t>((N * K + 255) / 256, 148 * 64);
  dequant_mx_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(q.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>(),
                                                                            N, (int)K, fp4 ? 1 : 0, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k
