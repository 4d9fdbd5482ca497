// Attention-side kernels for the hybrid models.
//
//  * qk_norm_rope_cache: per-head Gemma RMSNorm of q and k (x * rrms * (1 + w)), neox rotary
//    embedding on the first `rot` dims (partial RoPE), q written bf16, k and v quantised to e4m3
//    and scattered into the paged KV cache. Reference: kernels/r9k_norm_rope.hip:61 (norm + partial
//    rope) and the cache write of the stock attention backend.
//  * paged_attention: causal attention of a batch of query tokens against a paged fp8 KV cache.
//    Each query token is the last of `ctx` positions of its sequence; queries of one sequence
//    see earlier positions plus themselves (decode, spec verify and chunked prefill share it).
//    The attention-output gate (o * sigmoid(gate)) and the MXFP8 quantisation of the result for
//    the o_proj GEMM are fused into the final write. Reference: kernels/r9k_attn.hip:226-447.
//
// KV cache layout: [num_blocks][kv_heads][BLOCK=64][head_dim] e4m3 for K and V separately.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

constexpr int KV_BLOCK = 64;

// one warp per (token, head) row of length D (D % 32 == 0, D <= 512)
template <int D>
__global__ void qk_norm_rope_cache_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld_qkv, int Hq, int Hkv,
                                          int q_off, int k_off, int v_off, const __nv_bfloat16* __restrict__ qw,
                                          const __nv_bfloat16* __restrict__ kw, float eps, int plus_one,
                                          const int32_t* __restrict__ positions, const float* __restrict__ cos_sin,
                                          int rot, const int32_t* __restrict__ slots, __nv_bfloat16* __restrict__ q_out,
                                          uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache, float k_inv_scale,
                                          float v_inv_scale, int T) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  constexpr int PER = D / 32;
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int rows_per_tok = Hq + 2 * Hkv;
  if (gw >= (int64_t)T * rows_per_tok) return;
  const int t = (int)(gw / rows_per_tok);
  const int h = (int)(gw % rows_per_tok);
  const __nv_bfloat16* row = qkv + (int64_t)t * ld_qkv;
  int kind;  // 0 q, 1 k, 2 v
  int head;
  if (h < Hq) { kind = 0; head = h; }
  else if (h < Hq + Hkv) { kind = 1; head = h - Hq; }
  else { kind = 2; head = h - Hq - Hkv; }
  const __nv_bfloat16* src = row + (kind == 0 ? q_off + head * D : kind == 1 ? k_off + head * D : v_off + head * D);
  float x[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) x[i] = __bfloat162float(src[lane + 32 * i]);
  if (kind != 2) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) ss += x[i] * x[i];
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rr = rsqrtf(ss / (float)D + eps);
    const __nv_bfloat16* w = kind == 0 ? qw : kw;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      float wv = __bfloat162float(w[lane + 32 * i]);
      if (plus_one) wv += 1.f;
      x[i] = __bfloat162float(__float2bfloat16(x[i] * rr * wv));
    }
    // neox rotary on dims [0, rot): pairs (i, i + rot/2)
    if (rot > 0) {
      const int64_t pos = positions[t];
      const float* cs = cos_sin + pos * rot;  // [cos(rot/2) | sin(rot/2)]
      const int half = rot / 2;
      float y[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) y[i] = x[i];
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int d = lane + 32 * i;
        if (d < rot) {
          const int j = d < half ? d : d - half;
          const float c = cs[j], s = cs[half + j];
          // partner element d +- half lives in register i +- half/32 of the same lane when half % 32 == 0
          const int pi = d < half ? i + half / 32 : i - half / 32;
          const float partner = x[pi];
          y[i] = d < half ? x[i] * c - partner * s : x[i] * c + partner * s;
        }
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) x[i] = y[i];
    }
  }
  if (kind == 0) {
    __nv_bfloat16* dst = q_out + ((int64_t)t * Hq + head) * D;
#pragma unroll
    for (int i = 0; i < PER; ++i) dst[lane + 32 * i] = __float2bfloat16(x[i]);
  } else {
    const int64_t slot = slots[t];
    if (slot < 0) return;  // padding token
    const int64_t blk = slot / KV_BLOCK, off = slot % KV_BLOCK;
    uint8_t* dst = (kind == 1 ? k_cache : v_cache) + ((blk * Hkv + head) * KV_BLOCK + off) * D;
    const float inv = kind == 1 ? k_inv_scale : v_inv_scale;
#pragma unroll
    for (int i = 0; i < PER; ++i) dst[lane + 32 * i] = f32_to_e4m3(__bfloat162float(__float2bfloat16(x[i])) * inv);
  }
}

void qk_norm_rope_cache(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t q_off, int64_t k_off, int64_t v_off,
                        torch::Tensor qw, torch::Tensor kw, double eps, bool plus_one, torch::Tensor positions,
                        torch::Tensor cos_sin, int64_t rot, torch::Tensor slots, torch::Tensor q_out,
                        torch::Tensor k_cache, torch::Tensor v_cache, double k_scale, double v_scale) {
  const int64_t T = qkv.size(0);
  const int64_t D = q_out.size(-1);
  TORCH_CHECK(rot % 64 == 0 && rot <= D, "partial rope: rot must be a multiple of 64");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(qkv.device());
  const int64_t warps = T * (Hq + 2 * Hkv);
  const int threads = 256;
  const int blocks = (int)((warps * 32 + threads - 1) / threads);
  auto st = at::cuda::getCurrentCUDAStream();
#define R9K_QKNR(DD)                                                                                                 \
  launch_pdl(qk_norm_rope_cache_kernel<DD>, dim3(blocks), dim3(threads), 0, st,                                                         \
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), (int)Hq, (int)Hkv, (int)q_off, (int)k_off, \
      (int)v_off, reinterpret_cast<const __nv_bfloat16*>(qw.data_ptr()),                                             \
      reinterpret_cast<const __nv_bfloat16*>(kw.data_ptr()), (float)eps, plus_one ? 1 : 0,                           \
      positions.data_ptr<int32_t>(), cos_sin.data_ptr<float>(), (int)rot, slots.data_ptr<int32_t>(),                 \
      reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()), k_cache.data_ptr<uint8_t>(), v_cache.data_ptr<uint8_t>(),  \
      (float)(1.0 / k_scale), (float)(1.0 / v_scale), (int)T)
  if (D == 256) R9K_QKNR(256);
  else if (D == 128) R9K_QKNR(128);
  else TORCH_CHECK(false, "qk_norm_rope_cache: head_dim must be 128 or 256");
#undef R9K_QKNR
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------------------
// paged attention (CUDA cores). grid (T, Hq); 4 warps split the context; lane owns D/32 dims.
// ------------------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) paged_attention_kernel(
    const __nv_bfloat16* __restrict__ q, int Hq, int Hkv, const uint8_t* __restrict__ k_cache,
    const uint8_t* __restrict__ v_cache, const int32_t* __restrict__ block_table, int max_blocks,
    const int32_t* __restrict__ tok_seq, const int32_t* __restrict__ tok_ctx, float sm_scale, float k_scale,
    float v_scale, const __nv_bfloat16* __restrict__ gate, int64_t ld_gate, __nv_bfloat16* __restrict__ out,
    uint8_t* __restrict__ out_q, uint8_t* __restrict__ out_sf, int out_kblocks, int window) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  constexpr int PER = D / 32;
  const int t = blockIdx.x, h = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seq = tok_seq[t];
  const int ctx = tok_ctx[t];  // attend to positions [start, ctx)
  const int start = window > 0 ? max(0, ctx - window) : 0;
  const int kvh = h / (Hq / Hkv);
  float qv[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) qv[i] = __bfloat162float(q[((int64_t)t * Hq + h) * D + lane + 32 * i]) * sm_scale * k_scale;
  float m = -INFINITY, l = 0.f, acc[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) acc[i] = 0.f;
  const int32_t* bt = block_table + (int64_t)seq * max_blocks;
  for (int p = start + warp; p < ctx; p += 4) {
    const int64_t blk = bt[p / KV_BLOCK];
    const int64_t base = ((blk * Hkv + kvh) * KV_BLOCK + (p % KV_BLOCK)) * D;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) s += qv[i] * e4m3_to_f32(k_cache[base + lane + 32 * i]);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mn = fmaxf(m, s);
    const float corr = __expf(m - mn);
    const float pw = __expf(s - mn);
    l = l * corr + pw;
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] = acc[i] * corr + pw * e4m3_to_f32(v_cache[base + lane + 32 * i]);
    m = mn;
  }
  __shared__ float sm[4], sl[4], sacc[4][D];
  if (lane == 0) { sm[warp] = m; sl[warp] = l; }
#pragma unroll
  for (int i = 0; i < PER; ++i) sacc[warp][lane + 32 * i] = acc[i];
  __syncthreads();
  if (warp == 0) {
    float M = fmaxf(fmaxf(sm[0], sm[1]), fmaxf(sm[2], sm[3]));
    float L = 0.f, c[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) { c[w] = (sl[w] > 0.f) ? __expf(sm[w] - M) : 0.f; L += sl[w] * c[w]; }
    const float inv = L > 0.f ? v_scale / L : 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int d = lane + 32 * i;
      float o = (sacc[0][d] * c[0] + sacc[1][d] * c[1] + sacc[2][d] * c[2] + sacc[3][d] * c[3]) * inv;
      if (gate != nullptr) o *= sigmoid_f(__bfloat162float(gate[(int64_t)t * ld_gate + h * D + d]));
      o = __bfloat162float(__float2bfloat16(o));
      if (out != nullptr) out[((int64_t)t * Hq + h) * D + d] = __float2bfloat16(o);
      if (out_q != nullptr) {
        // MXFP8 block = 32 consecutive features = this warp's lanes for register i
        float am = fabsf(o);
        for (int s2 = 16; s2 > 0; s2 >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, s2));
        const int e = mx_exponent(am, 448.f);
        out_q[(int64_t)t * Hq * D + h * D + d] = f32_to_e4m3(o * exp2i(-e));
        if (lane == 0) out_sf[sf_offset(t, (h * D + 32 * i) >> 5, out_kblocks)] = (uint8_t)(e + 127);
      }
    }
  }
}

// Store new keys and values into the paged e4m3 cache by slot (slot = block * 64 + offset; negative
// slots are padding and skipped): one warp per (token, kv head), lane l handles elements l, l + 32, ...
__global__ void kv_cache_write_kernel(const __nv_bfloat16* __restrict__ k, int64_t ldk, const __nv_bfloat16* __restrict__ v,
                                      int64_t ldv, const int64_t* __restrict__ slots, int T, int Hkv, int D,
                                      uint8_t* __restrict__ kc, uint8_t* __restrict__ vc, float k_inv, float v_inv) {
  pdl_wait();
  pdl_trigger();
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)T * Hkv) return;
  const int t = (int)(gw / Hkv), h = (int)(gw % Hkv);
  const int64_t slot = slots[t];
  if (slot < 0) return;
  const int64_t blk = slot / KV_BLOCK, off = slot % KV_BLOCK;
  const int64_t dst = ((blk * Hkv + h) * KV_BLOCK + off) * D;
  const __nv_bfloat16* kr = k + (int64_t)t * ldk + (int64_t)h * D;
  const __nv_bfloat16* vr = v + (int64_t)t * ldv + (int64_t)h * D;
  for (int i = lane; i < D; i += 32) {
    kc[dst + i] = (uint8_t)__nv_cvt_float_to_fp8(__bfloat162float(kr[i]) * k_inv, __NV_SATFINITE, __NV_E4M3);
    vc[dst + i] = (uint8_t)__nv_cvt_float_to_fp8(__bfloat162float(vr[i]) * v_inv, __NV_SATFINITE, __NV_E4M3);
  }
}

void kv_cache_write(torch::Tensor k, torch::Tensor v, torch::Tensor slots, torch::Tensor k_cache,
                    torch::Tensor v_cache, double k_scale, double v_scale) {
  const int64_t T = k.size(0), Hkv = k.size(1), D = k.size(2);
  TORCH_CHECK(k.dtype() == torch::kBFloat16 && v.dtype() == torch::kBFloat16 && k.stride(2) == 1 && v.stride(2) == 1 &&
                  k.stride(1) == D && v.stride(1) == D, "kv_cache_write: bf16 [T, Hkv, D] with contiguous heads");
  TORCH_CHECK(slots.dtype() == torch::kInt64 && slots.numel() >= T, "kv_cache_write: int64 slot per token");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(1) == Hkv && k_cache.size(2) == KV_BLOCK && k_cache.size(3) == D &&
                  k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dtype() == torch::kUInt8,
              "kv_cache_write: caches uint8 [blocks, Hkv, 64, D]");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(k.device());
  const int64_t warps = T * Hkv;
  launch_pdl(kv_cache_write_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0,
             at::cuda::getCurrentCUDAStream(), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()), k.stride(0),
             reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), v.stride(0), slots.data_ptr<int64_t>(), (int)T,
             (int)Hkv, (int)D, k_cache.data_ptr<uint8_t>(), v_cache.data_ptr<uint8_t>(), (float)(1.0 / k_scale),
             (float)(1.0 / v_scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void paged_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                     torch::Tensor tok_seq, torch::Tensor tok_ctx, double sm_scale, double k_scale, double v_scale,
                     c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> out,
                     c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_sf, int64_t window) {
  const int64_t T = q.size(0), Hq = q.size(1), D = q.size(2);
  const int64_t Hkv = k_cache.size(1);
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const __nv_bfloat16* g = (gate.has_value() && gate->defined()) ? reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr()) : nullptr;
  const int64_t ldg = g ? gate->stride(0) : 0;
  __nv_bfloat16* o = (out.has_value() && out->defined()) ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  uint8_t* oq = (out_q.has_value() && out_q->defined()) ? out_q->data_ptr<uint8_t>() : nullptr;
  uint8_t* osf = (out_sf.has_value() && out_sf->defined()) ? out_sf->data_ptr<uint8_t>() : nullptr;
  dim3 grid((unsigned)T, (unsigned)Hq);
#define R9K_PA(DD)                                                                                                   \
  launch_pdl(paged_attention_kernel<DD>, grid, dim3(128), 0, st,                                                                  \
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), (int)Hq, (int)Hkv, k_cache.data_ptr<uint8_t>(),          \
      v_cache.data_ptr<uint8_t>(), block_table.data_ptr<int32_t>(), (int)block_table.size(1),                       \
      tok_seq.data_ptr<int32_t>(), tok_ctx.data_ptr<int32_t>(), (float)sm_scale, (float)k_scale, (float)v_scale, g,   \
      ldg, o, oq, osf, (int)(Hq * D / 32), (int)window)
  if (D == 256) R9K_PA(256);
  else if (D == 128) R9K_PA(128);
  else TORCH_CHECK(false, "paged_attention: head_dim must be 128 or 256");
#undef R9K_PA
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k
