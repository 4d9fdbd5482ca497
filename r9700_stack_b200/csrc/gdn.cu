// Gated DeltaNet (linear attention) kernels.
//
// Per value head h (key head h / (Hv/Hk)), per token:
//   g    = -exp(A_log[h]) * softplus(a + dt_bias[h])        beta = sigmoid(b)
//   q, k = l2norm(q) * dk^-1/2, l2norm(k)
//   S    = S * exp(g);  delta = beta * (v - S^T k);  S += k (x) delta;  o = S^T q
//   out  = rmsnorm(o) * w * silu(z)
// (reference: kernels/r9k_gdn.hip:4-21, :90-647; the reference's long prefill path calls stock
// Triton, r9700_vllm/models/gdn.py:28-33, which has no counterpart here: the recurrent core below
// serves prefill too.)
//
// Kernels:
//  * gdn_conv_prep      - causal depthwise conv1d (width W) over the q|k|v channels + SiLU, l2-norms,
//                         g and beta; reads the per-sequence conv state for the first W-1 taps.
//  * gdn_conv_state_update - stores the last W-1 conv inputs of each sequence (skipped during spec
//                         verify, run on commit).
//  * gdn_recurrent      - the delta-rule recurrence (state stored transposed, [dv][dk] per head).
//                         Columns of S evolve independently, so the grid
//                         splits each head's dv columns over CTAs (16 per CTA); eight lanes share a
//                         column (16 rows each) and reduce with shuffles, one reduction per token
//                         (the output dot and the next key dot share it), no block barrier per
//                         token. Serves decode (1 token), spec verify (T tokens, state not written),
//                         commit (accepted tokens, state written) and prefill.
//  * gdn_out_norm_quant - RMSNormGated + MXFP8 quantisation of the result for out_proj.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

template <typename T> R9K_DEVINL float to_f(T v);
template <> R9K_DEVINL float to_f<float>(float v) { return v; }
template <> R9K_DEVINL float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> R9K_DEVINL T from_f(float v);
template <> R9K_DEVINL float from_f<float>(float v) { return v; }
template <> R9K_DEVINL __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

// ------------------------------------------------------------------------------------------------
// conv + prep: grid (T, ceil((2*Hk + Hv + 1) / 8)), 8 warps; warp w handles 128-channel head
// hh = blockIdx.y * 8 + w of [q heads | k heads | v heads], the last index computes g and beta.
// Lane l owns channels 4l..4l+3 of the head. Requires dk == dv == 128.
// ------------------------------------------------------------------------------------------------
template <typename ST>
__global__ void gdn_conv_prep_kernel(const __nv_bfloat16* __restrict__ proj, int64_t ld, int Hk, int Hv, int dk,
                                     int dv, int b_off, int a_off, const __nv_bfloat16* __restrict__ conv_w, int W,
                                     const ST* __restrict__ conv_state, const int32_t* __restrict__ tok_slot,
                                     const int32_t* __restrict__ tok_pos_in_chunk,
                                     const int32_t* __restrict__ has_state_tok, const float* __restrict__ A_log,
                                     const float* __restrict__ dt_bias, float* __restrict__ q_out,
                                     float* __restrict__ k_out, float* __restrict__ v_out, float* __restrict__ g_out,
                                     float* __restrict__ beta_out, __nv_bfloat16* __restrict__ qkv_bf16) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int hh = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int NH = 2 * Hk + Hv;
  if (hh > NH) return;
  if (hh == NH) {
    for (int h = lane; h < Hv; h += 32) {
      const float av = __bfloat162float(proj[(int64_t)t * ld + a_off + h]);
      const float bv = __bfloat162float(proj[(int64_t)t * ld + b_off + h]);
      g_out[(int64_t)t * Hv + h] = -__expf(A_log[h]) * softplus_f(av + dt_bias[h]);
      beta_out[(int64_t)t * Hv + h] = sigmoid_f(bv);
    }
    return;
  }
  const int C = 2 * Hk * dk + Hv * dv;
  const int c0 = hh * 128 + lane * 4;
  const int j = tok_pos_in_chunk[t];
  const int slot = tok_slot[t];
  const bool hs = has_state_tok[t] != 0;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  // weights: 4 channels x W taps, contiguous
  float wt[4][8];
#pragma unroll
  for (int e = 0; e < 4; ++e)
    for (int w = 0; w < W; ++w) wt[e][w] = __bfloat162float(conv_w[(int64_t)(c0 + e) * W + w]);
  for (int w = 0; w < W; ++w) {
    const int back = W - 1 - w;
    float x[4];
    if (j - back >= 0) {
      const uint2 raw = *reinterpret_cast<const uint2*>(proj + (int64_t)(t - back) * ld + c0);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] = __bfloat162float(e[k]);
    } else {
      const int si = (W - 1) - (back - j);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        x[k] = (hs && si >= 0) ? to_f<ST>(conv_state[((int64_t)slot * C + c0 + k) * (W - 1) + si]) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] += x[k] * wt[k][w];
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) acc[k] = silu_f(acc[k]);
  if (hh < 2 * Hk) {
    float ss = acc[0] * acc[0] + acc[1] * acc[1] + acc[2] * acc[2] + acc[3] * acc[3];
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    float inv = rsqrtf(ss + 1e-6f);
    float* dst;
    if (hh < Hk) { inv *= rsqrtf((float)dk); dst = q_out + ((int64_t)t * Hk + hh) * dk; }
    else dst = k_out + ((int64_t)t * Hk + (hh - Hk)) * dk;
    *reinterpret_cast<float4*>(dst + lane * 4) = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] *= inv;
  } else {
    float* dst = v_out + ((int64_t)t * Hv + (hh - 2 * Hk)) * dv;
    *reinterpret_cast<float4*>(dst + lane * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
  if (qkv_bf16 != nullptr) {
    // [T, 2 Hk + Hv, 128] bf16 copy (q | k | v heads) for the chunked prefill's tensor-core tiles
    const __nv_bfloat162 lo = __floats2bfloat162_rn(acc[0], acc[1]), hi = __floats2bfloat162_rn(acc[2], acc[3]);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&lo);
    pk.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(qkv_bf16 + ((int64_t)t * NH + hh) * 128 + lane * 4) = pk;
  }
}

// state update: one CTA per sequence. The new state holds the last W-1 inputs of (old state ++ chunk).
template <typename ST>
__global__ void gdn_conv_state_update_kernel(const __nv_bfloat16* __restrict__ proj, int64_t ld, int C, int W,
                                             ST* __restrict__ conv_state, const int32_t* __restrict__ seq_slot,
                                             const int32_t* __restrict__ seq_start, const int32_t* __restrict__ seq_len,
                                             const int32_t* __restrict__ seq_has_state) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  const int s = blockIdx.x;
  const int slot = seq_slot[s], st0 = seq_start[s], n = seq_len[s];
  const bool hs = seq_has_state[s] != 0;
  if (n <= 0) return;
  {
    const int c = blockIdx.y * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float nv[8];
    ST* cs = conv_state + ((int64_t)slot * C + c) * (W - 1);
    for (int i = 0; i < W - 1; ++i) {
      // element i of the new state is input (n - (W-1) + i) of the concatenation old ++ chunk
      const int idx = n - (W - 1) + i;
      if (idx >= 0) nv[i] = __bfloat162float(proj[(int64_t)(st0 + idx) * ld + c]);
      else {
        const int oi = (W - 1) + idx;
        nv[i] = (hs && oi >= 0) ? to_f<ST>(cs[oi]) : 0.f;
      }
    }
    for (int i = 0; i < W - 1; ++i) cs[i] = from_f<ST>(nv[i]);
  }
}

// ------------------------------------------------------------------------------------------------
// recurrent core: grid (num_seqs, Hv, dv / 32), 128 threads. The state is stored transposed,
// [slot][h][dv][dk], so thread tid (column c = tid / 4 of this CTA's 32, row group rg = tid % 4)
// owns 32 contiguous dk entries of its column and moves them with 16-byte vectors.
// k/q are staged in smem interleaved as [token][r * 4 + rg] (row i = rg * 32 + r): conflict-free.
// ------------------------------------------------------------------------------------------------
template <typename ST> struct StateVec;
template <> struct StateVec<float> {
  R9K_DEVINL static void load(const float* p, float* v) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = reinterpret_cast<const float4*>(p)[i];
      v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
  }
  R9K_DEVINL static void store(float* p, const float* v) {
#pragma unroll
    for (int i = 0; i < 8; ++i) reinterpret_cast<float4*>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
};
template <> struct StateVec<__nv_bfloat16> {
  R9K_DEVINL static void load(const __nv_bfloat16* p, float* v) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 raw = reinterpret_cast<const uint4*>(p)[i];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[8 * i + k] = __bfloat162float(e[k]);
    }
  }
  R9K_DEVINL static void store(__nv_bfloat16* p, const float* v) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 raw;
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = __float2bfloat16(v[8 * i + k]);
      reinterpret_cast<uint4*>(p)[i] = raw;
    }
  }
};

template <typename ST> struct StateVec16;
template <> struct StateVec16<float> {
  R9K_DEVINL static void load(const float* p, float* v) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = reinterpret_cast<const float4*>(p)[i];
      v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
  }
  R9K_DEVINL static void store(float* p, const float* v) {
#pragma unroll
    for (int i = 0; i < 4; ++i) reinterpret_cast<float4*>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
};
template <> struct StateVec16<__nv_bfloat16> {
  R9K_DEVINL static void load(const __nv_bfloat16* p, float* v) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 raw = reinterpret_cast<const uint4*>(p)[i];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[8 * i + k] = __bfloat162float(e[k]);
    }
  }
  R9K_DEVINL static void store(__nv_bfloat16* p, const float* v) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint4 raw;
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = __float2bfloat16(v[8 * i + k]);
      reinterpret_cast<uint4*>(p)[i] = raw;
    }
  }
};

R9K_DEVINL void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
R9K_DEVINL void cp_async_4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// waits until at most n of this thread's cp.async groups are still in flight (n < 8)
R9K_DEVINL void cp_async_wait_pending(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
  }
}

// Token-serial delta rule. CTA = (sequence, value head, 16 state columns), 128 threads: lane
// (column cl, row group rg) of a warp owns 16 dk rows of one column, so 8 lanes share a column and
// reduce with three xor shuffles. The critical path per token is one shuffle reduction: the output
// dot S_t . q_t and the next token's key dot S_t . k_{t+1} read the same updated state and reduce
// together. q / k / v / g / beta are staged CH tokens at a time with cp.async into two buffers, the
// next chunk landing while this one runs.
template <typename ST, int DK>
__global__ void __launch_bounds__(128) gdn_recurrent_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta, int Hk, int Hv, int dv, ST* __restrict__ state,
    const int32_t* __restrict__ seq_slot, const int32_t* __restrict__ seq_start, const int32_t* __restrict__ seq_len,
    const int32_t* __restrict__ seq_has_state, int write_state, float* __restrict__ o) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  static_assert(DK == 128, "8 row groups of 16");
  constexpr int CH = 16, RPL = 16, RS = RPL + 4;  // RS: row-group stride (conflict-free 16-byte reads)
  __shared__ __align__(16) float sq[2][CH][8][RS];
  __shared__ __align__(16) float sk[2][CH][8][RS];
  __shared__ __align__(16) float sv[2][CH][16];
  __shared__ float sg[2][CH], sb[2][CH];
  const int s = blockIdx.x, h = blockIdx.y, cs = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31;
  const int rg = lane & 7, cl = ((tid >> 5) << 2) | (lane >> 3);
  const int col = cs * 16 + cl;
  const int kh = h / (Hv / Hk);
  const int slot = seq_slot[s], t0 = seq_start[s], n = seq_len[s];
  if (n <= 0 && !write_state) return;
  ST* Sp = state + (((int64_t)slot * Hv + h) * dv + col) * DK + rg * RPL;
  float S[RPL];
  if (seq_has_state[s] != 0) StateVec16<ST>::load(Sp, S);
  else {
#pragma unroll
    for (int r = 0; r < RPL; ++r) S[r] = 0.f;
  }
  auto stage = [&](int buf, int base) {
    const int cnt = min(CH, n - base);
    for (int e = tid; e < cnt * 32; e += 128) {
      const int tt = e >> 5, pc = e & 31;
      const int64_t off = ((int64_t)(t0 + base + tt) * Hk + kh) * DK + pc * 4;
      cp_async_16(&sq[buf][tt][pc >> 2][(pc & 3) * 4], q + off);
      cp_async_16(&sk[buf][tt][pc >> 2][(pc & 3) * 4], k + off);
    }
    if (tid < cnt * 4) {
      const int tt = tid >> 2, pc = tid & 3;
      cp_async_16(&sv[buf][tt][pc * 4], v + ((int64_t)(t0 + base + tt) * Hv + h) * dv + cs * 16 + pc * 4);
    }
    if (tid >= 64 && tid < 64 + cnt) {
      const int64_t tok = t0 + base + (tid - 64);
      cp_async_4(&sg[buf][tid - 64], g + tok * Hv + h);
      cp_async_4(&sb[buf][tid - 64], beta + tok * Hv + h);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  auto ld16 = [&](const float* p, float* x) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = reinterpret_cast<const float4*>(p)[i];
      x[4 * i] = f.x; x[4 * i + 1] = f.y; x[4 * i + 2] = f.z; x[4 * i + 3] = f.w;
    }
  };
  if (n > 0) {
    stage(0, 0);
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    float kc[RPL];
    ld16(&sk[0][0][rg][0], kc);
    float kv;
    {
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int r = 0; r < RPL; r += 4) {
        a0 += S[r] * kc[r]; a1 += S[r + 1] * kc[r + 1]; a2 += S[r + 2] * kc[r + 2]; a3 += S[r + 3] * kc[r + 3];
      }
      kv = (a0 + a1) + (a2 + a3);
      kv += __shfl_xor_sync(0xffffffffu, kv, 1);
      kv += __shfl_xor_sync(0xffffffffu, kv, 2);
      kv += __shfl_xor_sync(0xffffffffu, kv, 4);
    }
    for (int base = 0; base < n; base += CH) {
      const int buf = (base / CH) & 1;
      const int cnt = min(CH, n - base);
      const bool has_next_chunk = base + CH < n;
      if (has_next_chunk) stage(buf ^ 1, base + CH);
#pragma unroll 1
      for (int tt = 0; tt < cnt; ++tt) {
        const float decay = __expf(sg[buf][tt]), bt = sb[buf][tt], vt = sv[buf][tt][cl];
        float qv[RPL], kn[RPL];
        ld16(&sq[buf][tt][rg][0], qv);
        const bool last = tt == cnt - 1;
        const bool more = !last || has_next_chunk;
        if (!last) {
          ld16(&sk[buf][tt + 1][rg][0], kn);
        } else {
          // the next chunk has landed and every thread is done with this buffer past this point
          asm volatile("cp.async.wait_all;" ::: "memory");
          __syncthreads();
          if (more) ld16(&sk[buf ^ 1][0][rg][0], kn);
        }
        const float delta = bt * (vt - decay * kv);
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f, k0 = 0.f, k1 = 0.f, k2 = 0.f, k3 = 0.f;
#pragma unroll
        for (int r = 0; r < RPL; r += 4) {
          S[r] = S[r] * decay + kc[r] * delta;
          S[r + 1] = S[r + 1] * decay + kc[r + 1] * delta;
          S[r + 2] = S[r + 2] * decay + kc[r + 2] * delta;
          S[r + 3] = S[r + 3] * decay + kc[r + 3] * delta;
          o0 += S[r] * qv[r]; o1 += S[r + 1] * qv[r + 1]; o2 += S[r + 2] * qv[r + 2]; o3 += S[r + 3] * qv[r + 3];
          if (more) {
            k0 += S[r] * kn[r]; k1 += S[r + 1] * kn[r + 1]; k2 += S[r + 2] * kn[r + 2]; k3 += S[r + 3] * kn[r + 3];
          }
        }
        float ov = (o0 + o1) + (o2 + o3), kvn = (k0 + k1) + (k2 + k3);
#pragma unroll
        for (int m = 1; m <= 4; m <<= 1) {
          ov += __shfl_xor_sync(0xffffffffu, ov, m);
          kvn += __shfl_xor_sync(0xffffffffu, kvn, m);
        }
        if (o != nullptr && rg == 0) o[((int64_t)(t0 + base + tt) * Hv + h) * dv + col] = ov;
        kv = kvn;
        if (more) {
#pragma unroll
          for (int r = 0; r < RPL; ++r) kc[r] = kn[r];
        }
      }
    }
  }
  if (write_state) StateVec16<ST>::store(Sp, S);
}

// ------------------------------------------------------------------------------------------------
// RMSNormGated + MXFP8: one warp per (token, head), dv = 128 (4 elements per lane)
// ------------------------------------------------------------------------------------------------
__global__ void gdn_out_norm_quant_kernel(const float* __restrict__ o, const __nv_bfloat16* __restrict__ proj,
                                          int64_t ld, int z_off, const __nv_bfloat16* __restrict__ w, float eps,
                                          int T, int Hv, int dv, __nv_bfloat16* __restrict__ y,
                                          uint8_t* __restrict__ out_q, uint8_t* __restrict__ out_sf) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  pdl_trigger();  // the next GEMM may start streaming its weights
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)T * Hv) return;
  const int t = (int)(gw / Hv), h = (int)(gw % Hv);
  const int per = dv / 32;
  float x[8];
  float ss = 0.f;
  for (int i = 0; i < per; ++i) {
    x[i] = o[((int64_t)t * Hv + h) * dv + lane + 32 * i];
    ss += x[i] * x[i];
  }
  for (int s2 = 16; s2 > 0; s2 >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s2);
  const float rr = rsqrtf(ss / (float)dv + eps);
  const int kblocks = Hv * dv / 32;
  for (int i = 0; i < per; ++i) {
    const int d = lane + 32 * i;
    const float z = __bfloat162float(proj[(int64_t)t * ld + z_off + h * dv + d]);
    float val = x[i] * rr * __bfloat162float(w[d]) * silu_f(z);
    val = __bfloat162float(__float2bfloat16(val));
    if (y != nullptr) y[((int64_t)t * Hv + h) * dv + d] = __float2bfloat16(val);
    if (out_q != nullptr) {
      float am = fabsf(val);
      for (int s2 = 16; s2 > 0; s2 >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, s2));
      const int e = mx_exponent(am, 448.f);
      out_q[(int64_t)t * Hv * dv + h * dv + d] = f32_to_e4m3(val * exp2i(-e));
      if (lane == 0) out_sf[sf_offset(t, (h * dv + 32 * i) >> 5, kblocks)] = (uint8_t)(e + 127);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// host wrappers
// ------------------------------------------------------------------------------------------------
void gdn_conv_prep(torch::Tensor proj, int64_t Hk, int64_t Hv, int64_t dk, int64_t dv, int64_t b_off, int64_t a_off,
                   torch::Tensor conv_w, torch::Tensor conv_state, torch::Tensor tok_slot, torch::Tensor tok_pos,
                   torch::Tensor tok_has_state, torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor q_out,
                   torch::Tensor k_out, torch::Tensor v_out, torch::Tensor g_out, torch::Tensor beta_out,
                   c10::optional<torch::Tensor> qkv_bf16) {
  const int64_t T = proj.size(0);
  if (T == 0) return;
  __nv_bfloat16* qb = nullptr;
  if (qkv_bf16.has_value() && qkv_bf16->defined()) {
    TORCH_CHECK(qkv_bf16->dtype() == torch::kBFloat16 && qkv_bf16->is_contiguous() &&
                    qkv_bf16->numel() >= T * (2 * Hk + Hv) * 128,
                "gdn_conv_prep: qkv_bf16 [T, 2 Hk + Hv, 128] bf16");
    qb = reinterpret_cast<__nv_bfloat16*>(qkv_bf16->data_ptr());
  }
  const int64_t C = 2 * Hk * dk + Hv * dv;
  const int W = (int)conv_w.size(1);
  TORCH_CHECK(conv_state.size(-1) == W - 1 && conv_state.size(1) == C, "gdn_conv_prep: conv state shape");
  const at::cuda::CUDAGuard guard(proj.device());
  auto st = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(dk == 128 && dv == 128 && W <= 8, "gdn_conv_prep: head dim 128, conv width <= 8");
  TORCH_CHECK(proj.stride(0) % 4 == 0 && proj.stride(1) == 1, "gdn_conv_prep: proj rows must be 8-byte aligned");
  const dim3 grid((unsigned)T, (unsigned)((2 * Hk + Hv + 1 + 7) / 8));
#define R9K_CONV(ST_T)                                                                                                \
  launch_pdl(gdn_conv_prep_kernel<ST_T>, grid, dim3(256), 0, st,                                                                    \
      reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), proj.stride(0), (int)Hk, (int)Hv, (int)dk, (int)dv,     \
      (int)b_off, (int)a_off, reinterpret_cast<const __nv_bfloat16*>(conv_w.data_ptr()), W,                           \
      reinterpret_cast<const ST_T*>(conv_state.data_ptr()), tok_slot.data_ptr<int32_t>(), tok_pos.data_ptr<int32_t>(),  \
      tok_has_state.data_ptr<int32_t>(), A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), q_out.data_ptr<float>(),  \
      k_out.data_ptr<float>(), v_out.data_ptr<float>(), g_out.data_ptr<float>(), beta_out.data_ptr<float>(), qb);
  if (conv_state.dtype() == torch::kFloat32) { R9K_CONV(float) } else { R9K_CONV(__nv_bfloat16) }
#undef R9K_CONV
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_conv_state_update(torch::Tensor proj, torch::Tensor conv_state, torch::Tensor seq_slot,
                           torch::Tensor seq_start, torch::Tensor seq_len, torch::Tensor seq_has_state) {
  const int64_t S = seq_slot.size(0);
  if (S == 0) return;
  const int C = (int)conv_state.size(1);
  const int W = (int)conv_state.size(2) + 1;
  TORCH_CHECK(W - 1 <= 8, "conv width <= 9");
  const at::cuda::CUDAGuard guard(proj.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const dim3 grid((unsigned)S, (unsigned)((C + 255) / 256));
  if (conv_state.dtype() == torch::kFloat32)
    launch_pdl(gdn_conv_state_update_kernel<float>, grid, dim3(256), 0, st,
        reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), proj.stride(0), C, W, conv_state.data_ptr<float>(),
        seq_slot.data_ptr<int32_t>(), seq_start.data_ptr<int32_t>(), seq_len.data_ptr<int32_t>(),
        seq_has_state.data_ptr<int32_t>());
  else
    launch_pdl(gdn_conv_state_update_kernel<__nv_bfloat16>, grid, dim3(256), 0, st,
        reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), proj.stride(0), C, W,
        reinterpret_cast<__nv_bfloat16*>(conv_state.data_ptr()), seq_slot.data_ptr<int32_t>(),
        seq_start.data_ptr<int32_t>(), seq_len.data_ptr<int32_t>(), seq_has_state.data_ptr<int32_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_recurrent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                   torch::Tensor state, torch::Tensor seq_slot, torch::Tensor seq_start, torch::Tensor seq_len,
                   torch::Tensor seq_has_state, bool write_state, c10::optional<torch::Tensor> o) {
  const int64_t S = seq_slot.size(0);
  if (S == 0) return;
  const int Hk = (int)q.size(1), DK = (int)q.size(2);
  const int Hv = (int)v.size(1), dv = (int)v.size(2);
  TORCH_CHECK(dv % 16 == 0 && DK == 128, "gdn_recurrent: dk 128, dv % 16");
  TORCH_CHECK(state.size(1) == Hv && state.size(2) == dv && state.size(3) == DK, "gdn_recurrent: state [slots, Hv, dv, dk]");
  const at::cuda::CUDAGuard guard(q.device());
  auto st = at::cuda::getCurrentCUDAStream();
  dim3 grid((unsigned)S, (unsigned)Hv, (unsigned)(dv / 16));
  float* op = (o.has_value() && o->defined()) ? o->data_ptr<float>() : nullptr;
  if (state.dtype() == torch::kFloat32)
    launch_pdl(gdn_recurrent_kernel<float, 128>, grid, dim3(128), 0, st,
        q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), g.data_ptr<float>(), beta.data_ptr<float>(), Hk,
        Hv, dv, state.data_ptr<float>(), seq_slot.data_ptr<int32_t>(), seq_start.data_ptr<int32_t>(),
        seq_len.data_ptr<int32_t>(), seq_has_state.data_ptr<int32_t>(), write_state ? 1 : 0, op);
  else
    launch_pdl(gdn_recurrent_kernel<__nv_bfloat16, 128>, grid, dim3(128), 0, st,
        q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), g.data_ptr<float>(), beta.data_ptr<float>(), Hk,
        Hv, dv, reinterpret_cast<__nv_bfloat16*>(state.data_ptr()), seq_slot.data_ptr<int32_t>(),
        seq_start.data_ptr<int32_t>(), seq_len.data_ptr<int32_t>(), seq_has_state.data_ptr<int32_t>(),
        write_state ? 1 : 0, op);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_out_norm_quant(torch::Tensor o, torch::Tensor proj, int64_t z_off, torch::Tensor w, double eps,
                        c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> out_q,
                        c10::optional<torch::Tensor> out_sf) {
  const int64_t T = o.size(0), Hv = o.size(1), dv = o.size(2);
  if (T == 0) return;
  TORCH_CHECK(dv % 32 == 0 && dv <= 256, "gdn_out_norm_quant: dv");
  const at::cuda::CUDAGuard guard(o.device());
  const int64_t warps = T * Hv;
  const int blocks = (int)((warps * 32 + 255) / 256);
  launch_pdl(gdn_out_norm_quant_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
      o.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), proj.stride(0), (int)z_off,
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (float)eps, (int)T, (int)Hv, (int)dv,
      (y.has_value() && y->defined()) ? reinterpret_cast<__nv_bfloat16*>(y->data_ptr()) : nullptr,
      (out_q.has_value() && out_q->defined()) ? out_q->data_ptr<uint8_t>() : nullptr,
      (out_sf.has_value() && out_sf->defined()) ? out_sf->data_ptr<uint8_t>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k

namespace r9k {

// ------------------------------------------------------------------------------------------------
// Fused decode step (every sequence contributes exactly one token): one CTA per (sequence, key head)
// does the causal conv (and conv-state update) of the key head's q/k channels and of its `rep` value
// heads, the l2-norms and gates, then for each value head the delta-rule update (state read and
// written once), RMSNormGated and the MXFP8 quantisation of the output for out_proj.
// The CTA owns every conv channel it touches, so no other CTA reads state it writes.
// 512 threads: recurrence thread (c = tid / 4, rg = tid % 4) owns 32 contiguous dk rows of column c.
// ------------------------------------------------------------------------------------------------
template <typename ST>
__global__ void __launch_bounds__(512, 2) gdn_decode_fused_kernel(
    const __nv_bfloat16* __restrict__ proj, int64_t ld, int Hk, int Hv, int z_off, int b_off, int a_off,
    const __nv_bfloat16* __restrict__ conv_w, ST* __restrict__ conv_state, ST* __restrict__ state,
    const int32_t* __restrict__ seq_slot, const int32_t* __restrict__ seq_has_state, const float* __restrict__ A_log,
    const float* __restrict__ dt_bias, const __nv_bfloat16* __restrict__ norm_w, float eps,
    uint8_t* __restrict__ out_q, uint8_t* __restrict__ out_sf, __nv_bfloat16* __restrict__ out_bf16) {
  // grid (sequence, key head): the CTA owns the key head's q / k channels and its rep value heads,
  // so it updates all of their conv state itself. Every value head's state (128 x 128) is requested
  // with asynchronous copies before anything else (rep x 32 KB in flight per CTA for bf16 state),
  // then the heads are updated one after another out of shared memory.
  // Thread (column c = tid / 4, quarter rg = tid % 4) owns 32 entries of a column per head.
  constexpr int D = 128, W = 4, PER = 32, PC = 16, MAXREP = 8, NT = 512, NG = D / PER;
  __shared__ float sq[NG][PER + 1], sk[NG][PER + 1];  // [quarter][row]: quarters sit in different banks
  __shared__ float sv[MAXREP][D], so[4][D], sred[2][16];
  __shared__ float sg[MAXREP], sb[MAXREP];
  extern __shared__ __align__(16) uint8_t s_state[];
  const int t = blockIdx.x, kh = blockIdx.y;
  const int rep = Hv / Hk;
  const int tid = threadIdx.x;
  const int C = 2 * Hk * D + Hv * D;
  const int slot = seq_slot[t];  // step metadata: copied in before the forward began
  const bool hs = seq_has_state[t] != 0;
  const int c = tid >> 2, rg = tid & 3;
  constexpr int NV = PER * sizeof(ST) / 16;  // 16-byte chunks per thread and head
  uint4* sS = reinterpret_cast<uint4*>(s_state);
  // chunk v of thread tid for head j at (j * NV + v) * NT + tid: conflict-free
  // one cp.async group per value head: head j waits only for its own state (each thread reads back
  // exactly the chunks it requested, so no block barrier is needed for them)
  if (hs) {
    for (int j = 0; j < rep; ++j) {
      const ST* Sp = state + (((int64_t)slot * Hv + kh * rep + j) * D + c) * D + rg * PER;
#pragma unroll
      for (int v = 0; v < NV; ++v)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sS + (j * NV + v) * NT + tid)),
                     "l"(reinterpret_cast<const uint8_t*>(Sp) + 16 * v) : "memory");
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
  }
  // ---- conv over q (128) | k (128) | the rep value heads (rep x 128) channels. The conv state (last
  // written by this layer's previous step) and the conv weights do not depend on the preceding grid:
  // they are read into registers before waiting on it; only the new projection row comes after.
  constexpr int MAXCH = ((2 + MAXREP) * D + NT - 1) / NT;
  const int nch = (2 + rep) * D;
  auto chan = [&](int ch) {
    const int part = ch / D, i = ch % D;
    return part == 0 ? kh * D + i : part == 1 ? Hk * D + kh * D + i : 2 * Hk * D + (kh * rep + part - 2) * D + i;
  };
  float cst[MAXCH][W - 1], cwt[MAXCH][W];
#pragma unroll
  for (int u = 0; u < MAXCH; ++u) {
    const int ch = tid + u * NT;
    if (ch < nch) {
      const int cch = chan(ch);
      const ST* cs = conv_state + ((int64_t)slot * C + cch) * (W - 1);
#pragma unroll
      for (int w = 0; w < W - 1; ++w) cst[u][w] = hs ? to_f<ST>(cs[w]) : 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) cwt[u][w] = __bfloat162float(conv_w[(int64_t)cch * W + w]);
    }
  }
  pdl_wait();
  pdl_trigger();
#pragma unroll
  for (int u = 0; u < MAXCH; ++u) {
    const int ch = tid + u * NT;
    if (ch >= nch) break;
    const int part = ch / D, i = ch % D;
    const int cch = chan(ch);
    ST* cs = conv_state + ((int64_t)slot * C + cch) * (W - 1);
    float x[W];
#pragma unroll
    for (int w = 0; w < W - 1; ++w) x[w] = cst[u][w];
    x[W - 1] = __bfloat162float(proj[(int64_t)t * ld + cch]);
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) acc += x[w] * cwt[u][w];
#pragma unroll
    for (int w = 0; w < W - 1; ++w) cs[w] = from_f<ST>(x[w + 1]);
    const float y = silu_f(acc);
    if (part == 0) sq[i / PER][i % PER] = y;
    else if (part == 1) sk[i / PER][i % PER] = y;
    else sv[part - 2][i] = y;
  }
  if (tid < rep) {
    const int h = kh * rep + tid;
    const float av = __bfloat162float(proj[(int64_t)t * ld + a_off + h]);
    const float bv = __bfloat162float(proj[(int64_t)t * ld + b_off + h]);
    sg[tid] = __expf(-__expf(A_log[h]) * softplus_f(av + dt_bias[h]));  // decay factor exp(g)
    sb[tid] = sigmoid_f(bv);
  }
  __syncthreads();
  // ---- l2 norms of q and k (warps 0 and 1)
  if (tid < 64) {
    const float* src = tid < 32 ? &sq[0][0] : &sk[0][0];
    const int l = tid & 31;
    float ss = 0.f;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int i = l + 32 * jj;
      const float v = src[(i / PER) * (PER + 1) + i % PER];
      ss += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (l == 0) sred[0][tid >> 5] = rsqrtf(ss + 1e-6f);
  }
  __syncthreads();
  const float qs = sred[0][0] * rsqrtf((float)D), ks = sred[0][1];
  const float* kk = sk[rg];
  const float* qq = sq[rg];
  for (int j = 0; j < rep; ++j) {
    const int h = kh * rep + j;
    ST* Sp = state + (((int64_t)slot * Hv + h) * D + c) * D + rg * PER;
    const float decay = sg[j];
    if (hs) cp_async_wait_pending(rep - 1 - j);
    float kvs = 0.f;
#pragma unroll 1
    for (int p = 0; p < PER / PC; ++p) {
      float S[PC];
      if (hs) {
        constexpr int CPP = NV / (PER / PC);
        uint4 raw[CPP];
#pragma unroll
        for (int q = 0; q < CPP; ++q) raw[q] = sS[(j * NV + p * CPP + q) * NT + tid];
        StateVec16<ST>::load(reinterpret_cast<const ST*>(raw), S);
      } else {
#pragma unroll
        for (int r = 0; r < PC; ++r) S[r] = 0.f;
      }
#pragma unroll
      for (int r = 0; r < PC; ++r) kvs += S[r] * kk[p * PC + r];
    }
    kvs *= ks;
    kvs += __shfl_xor_sync(0xffffffffu, kvs, 1);
    kvs += __shfl_xor_sync(0xffffffffu, kvs, 2);
    const float delta = sb[j] * (sv[j][c] - decay * kvs);
    const float dk = delta * ks;
    float ov = 0.f;
#pragma unroll 1
    for (int p = 0; p < PER / PC; ++p) {
      float S[PC];
      if (hs) {
        constexpr int CPP = NV / (PER / PC);
        uint4 raw[CPP];
#pragma unroll
        for (int q = 0; q < CPP; ++q) raw[q] = sS[(j * NV + p * CPP + q) * NT + tid];
        StateVec16<ST>::load(reinterpret_cast<const ST*>(raw), S);
      } else {
#pragma unroll
        for (int r = 0; r < PC; ++r) S[r] = 0.f;
      }
#pragma unroll
      for (int r = 0; r < PC; ++r) {
        S[r] = S[r] * decay + kk[p * PC + r] * dk;
        ov += S[r] * qq[p * PC + r];
      }
      StateVec16<ST>::store(Sp + p * PC, S);
    }
    ov *= qs;
    ov += __shfl_xor_sync(0xffffffffu, ov, 1);
    ov += __shfl_xor_sync(0xffffffffu, ov, 2);
    const int gq = j & 3;  // the group of 128 threads that finishes this head
    if (rg == 0) so[gq][c] = ov;
    // ---- RMSNormGated + MXFP8 of this head: warps 4 gq .. 4 gq + 3 (column 32 * warp' + lane)
    __syncthreads();
    const int grp = (tid >> 7), tt = tid & 127;
    if (grp == gq) {
      const float o = so[gq][tt];
      float ss = o * o;
      for (int s2 = 16; s2 > 0; s2 >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s2);
      if ((tt & 31) == 0) sred[1][gq * 4 + (tt >> 5)] = ss;
      switch (gq) {
        case 0: asm volatile("bar.sync 1, 128;" ::: "memory"); break;
        case 1: asm volatile("bar.sync 2, 128;" ::: "memory"); break;
        case 2: asm volatile("bar.sync 3, 128;" ::: "memory"); break;
        default: asm volatile("bar.sync 4, 128;" ::: "memory"); break;
      }
      const float* sr = &sred[1][gq * 4];
      const float rr = rsqrtf((sr[0] + sr[1] + sr[2] + sr[3]) / (float)D + eps);
      const float z = __bfloat162float(proj[(int64_t)t * ld + z_off + h * D + tt]);
      float val = o * rr * __bfloat162float(norm_w[tt]) * silu_f(z);
      val = __bfloat162float(__float2bfloat16(val));
      const int64_t oi = (int64_t)t * Hv * D + h * D + tt;
      if (out_bf16 != nullptr) out_bf16[oi] = __float2bfloat16(val);
      if (out_q != nullptr) {
        float am = fabsf(val);
        for (int s2 = 16; s2 > 0; s2 >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, s2));
        const int e = mx_exponent(am, 448.f);
        out_q[oi] = f32_to_e4m3(val * exp2i(-e));
        if ((tt & 31) == 0) out_sf[sf_offset(t, (h * D + tt) >> 5, Hv * D / 32)] = (uint8_t)(e + 127);
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// L2 prefetch of the recurrent and conv state of the sequences in a decode step: launched in front of
// the layer's in_proj GEMM, it brings the state rows the fused GDN kernel will read into L2 while the
// GEMM streams its weights (evict-first), so the GDN kernel does not start with a 25 MB HBM read. A
// hint only: nothing reads its result. grid (sequences, pieces), 4 KiB per bulk prefetch.
// ------------------------------------------------------------------------------------------------
__global__ void gdn_state_prefetch_kernel(const uint8_t* __restrict__ state, int64_t state_row,
                                          const uint8_t* __restrict__ conv, int64_t conv_row,
                                          const int32_t* __restrict__ seq_slot) {
  pdl_trigger();  // the GEMM behind may launch at once; nothing here depends on the kernel before
  const int slot = seq_slot[blockIdx.x];
  constexpr int64_t PIECE = 4096;
  const uint8_t* sr = state + (int64_t)slot * state_row;
  for (int64_t o = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) * PIECE; o < state_row;
       o += (int64_t)gridDim.y * blockDim.x * PIECE) {
    const uint32_t n = (uint32_t)(state_row - o < PIECE ? state_row - o : PIECE);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(sr + o), "r"(n) : "memory");
  }
  if (blockIdx.y == 0 && conv != nullptr) {
    const uint8_t* cr = conv + (int64_t)slot * conv_row;
    for (int64_t o = (int64_t)threadIdx.x * PIECE; o < conv_row; o += (int64_t)blockDim.x * PIECE) {
      const uint32_t n = (uint32_t)(conv_row - o < PIECE ? conv_row - o : PIECE);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(cr + o), "r"(n) : "memory");
    }
  }
}

void gdn_state_prefetch(torch::Tensor state, c10::optional<torch::Tensor> conv_state, torch::Tensor seq_slot) {
  const int64_t S = seq_slot.size(0);
  if (S == 0) return;
  TORCH_CHECK(state.is_contiguous() && seq_slot.dtype() == torch::kInt32, "gdn_state_prefetch: state, int32 slots");
  const int64_t srow = state.numel() / state.size(0) * state.element_size();
  const bool has_conv = conv_state.has_value() && conv_state->defined();
  const int64_t crow = has_conv ? conv_state->numel() / conv_state->size(0) * conv_state->element_size() : 0;
  TORCH_CHECK(srow % 16 == 0 && crow % 16 == 0 && (reinterpret_cast<uintptr_t>(state.data_ptr()) & 15) == 0 &&
              (!has_conv || (reinterpret_cast<uintptr_t>(conv_state->data_ptr()) & 15) == 0),
              "gdn_state_prefetch: 16-byte rows");
  const at::cuda::CUDAGuard guard(state.device());
  const int pieces = (int)std::min<int64_t>(8, (srow / 4096 + 127) / 128);
  TORCH_CHECK(launch_pdl(gdn_state_prefetch_kernel, dim3((unsigned)S, (unsigned)std::max(1, pieces)), dim3(128), 0,
                         at::cuda::getCurrentCUDAStream(), reinterpret_cast<const uint8_t*>(state.data_ptr()), srow,
                         has_conv ? reinterpret_cast<const uint8_t*>(conv_state->data_ptr()) : nullptr, crow,
                         seq_slot.data_ptr<int32_t>()) == cudaSuccess,
              "gdn_state_prefetch launch");
}

void gdn_decode_fused(torch::Tensor proj, int64_t Hk, int64_t Hv, int64_t z_off, int64_t b_off, int64_t a_off,
                      torch::Tensor conv_w, torch::Tensor conv_state, torch::Tensor state, torch::Tensor seq_slot,
                      torch::Tensor seq_has_state, torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w,
                      double eps, c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_sf,
                      c10::optional<torch::Tensor> out_bf16) {
  const int64_t S = seq_slot.size(0);
  if (S == 0) return;
  TORCH_CHECK(proj.size(0) == S, "gdn_decode_fused: one token per sequence");
  TORCH_CHECK(conv_w.size(1) == 4 && Hv % Hk == 0 && Hv / Hk <= 8, "gdn_decode_fused: conv width 4, rep <= 8");
  TORCH_CHECK(state.size(2) == 128 && state.size(3) == 128, "gdn_decode_fused: head dim 128");
  const at::cuda::CUDAGuard guard(proj.device());
  const int rep = (int)(Hv / Hk);
  auto st = at::cuda::getCurrentCUDAStream();
  auto u8 = [](const c10::optional<torch::Tensor>& t) -> uint8_t* {
    return (t.has_value() && t->defined()) ? t->data_ptr<uint8_t>() : nullptr;
  };
  __nv_bfloat16* ob = (out_bf16.has_value() && out_bf16->defined()) ? reinterpret_cast<__nv_bfloat16*>(out_bf16->data_ptr()) : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)S, (unsigned)Hk, 1);
  cfg.blockDim = dim3(512);
  cfg.dynamicSmemBytes = (size_t)rep * 128 * 128 * state.element_size();
  TORCH_CHECK(cfg.dynamicSmemBytes <= 200 * 1024, "gdn_decode_fused: value heads per key head x state size exceed shared memory");
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
#define R9K_GDF(ST_T)                                                                                                 \
  {                                                                                                                   \
    ensure_smem_attr((const void*)gdn_decode_fused_kernel<ST_T>, 200 * 1024);                                       \
  }                                                                                                                   \
  TORCH_CHECK(cudaLaunchKernelEx(&cfg, gdn_decode_fused_kernel<ST_T>,                                                 \
      reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), proj.stride(0), (int)Hk, (int)Hv, (int)z_off, (int)b_off, \
      (int)a_off, reinterpret_cast<const __nv_bfloat16*>(conv_w.data_ptr()),                                          \
      reinterpret_cast<ST_T*>(conv_state.data_ptr()), reinterpret_cast<ST_T*>(state.data_ptr()),                      \
      seq_slot.data_ptr<int32_t>(), seq_has_state.data_ptr<int32_t>(), A_log.data_ptr<float>(),                        \
      dt_bias.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr()), (float)eps, u8(out_q),      \
      u8(out_sf), ob) == cudaSuccess, "gdn_decode_fused launch")
  if (state.dtype() == torch::kFloat32) { R9K_GDF(float); } else { R9K_GDF(__nv_bfloat16); }
#undef R9K_GDF
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------------------
// speculative commit: after a verify pass (state not written) accepted n_s tokens of sequence s;
// replay the recurrence over those tokens from the saved per-layer k/v/g/beta and store the state,
// and shift the conv state by the same tokens' saved inputs. All GDN layers in one launch:
// grid (S, Hv * dv/32 + ceil(C / 128), layers), 128 threads. CTAs y < Hv * dv/32 run the recurrence
// of (head, 32-column group) exactly as gdn_recurrent_kernel (without q / output); the others update
// 128 conv channels each. The two parts touch disjoint state, so they need no ordering.
// (reference: kernels/r9k_gdn.hip:575-647 r9k_gdn_spec_commit_kernel.)
// ------------------------------------------------------------------------------------------------
struct GdnCommitLayer {
  const float* k;     // [Tv, Hk, 128]
  const float* v;     // [Tv, Hv, dv]
  const float* g;     // [Tv, Hv] (log decay)
  const float* beta;  // [Tv, Hv]
  const __nv_bfloat16* proj;  // [Tv, ld]: conv inputs in the first C channels
  void* ssm;          // [slots, Hv, dv, 128]
  void* conv;         // [slots, C, W-1]
  int64_t pad;
};

template <typename ST>
__global__ void __launch_bounds__(128) gdn_spec_commit_kernel(
    const GdnCommitLayer* __restrict__ layers, int Hk, int Hv, int dv, int C, int W, int64_t ld,
    const int32_t* __restrict__ seq_slot, const int32_t* __restrict__ seq_start, const int32_t* __restrict__ acc_len,
    const int32_t* __restrict__ seq_has_state) {
  pdl_wait();
  pdl_trigger();
  constexpr int DK = 128, CH = 16;
  __shared__ float sk[CH][DK], sv[CH][32], sg[CH], sb[CH];
  const GdnCommitLayer Lr = layers[blockIdx.z];
  const int s = blockIdx.x, tid = threadIdx.x;
  const int slot = seq_slot[s], t0 = seq_start[s], n = acc_len[s];
  const bool hs = seq_has_state[s] != 0;
  if (n <= 0) return;
  const int nrec = Hv * (dv / 32);
  if ((int)blockIdx.y >= nrec) {
    const int c = ((int)blockIdx.y - nrec) * 128 + tid;
    if (c >= C) return;
    ST* cs = reinterpret_cast<ST*>(Lr.conv) + ((int64_t)slot * C + c) * (W - 1);
    float nv[8];
    for (int i = 0; i < W - 1; ++i) {
      const int idx = n - (W - 1) + i;
      if (idx >= 0) nv[i] = __bfloat162float(Lr.proj[(int64_t)(t0 + idx) * ld + c]);
      else {
        const int oi = (W - 1) + idx;
        nv[i] = (hs && oi >= 0) ? to_f<ST>(cs[oi]) : 0.f;
      }
    }
    for (int i = 0; i < W - 1; ++i) cs[i] = from_f<ST>(nv[i]);
    return;
  }
  const int h = (int)blockIdx.y / (dv / 32), cgrp = (int)blockIdx.y % (dv / 32);
  const int c = tid >> 2, rg = tid & 3;
  const int col = cgrp * 32 + c;
  const int kh = h / (Hv / Hk);
  ST* Sp = reinterpret_cast<ST*>(Lr.ssm) + (((int64_t)slot * Hv + h) * dv + col) * DK + rg * 32;
  float S[32];
  if (hs) StateVec<ST>::load(Sp, S);
  else {
#pragma unroll
    for (int r = 0; r < 32; ++r) S[r] = 0.f;
  }
  for (int base = 0; base < n; base += CH) {
    const int cnt = min(CH, n - base);
    __syncthreads();
    for (int e = tid; e < cnt * DK; e += 128) {
      const int tt = e / DK, i = e % DK;
      const int64_t tok = t0 + base + tt;
      sk[tt][(i & 31) * 4 + (i >> 5)] = Lr.k[(tok * Hk + kh) * DK + i];
    }
    for (int e = tid; e < cnt * 32; e += 128) {
      const int tt = e / 32, cc = e % 32;
      sv[tt][cc] = Lr.v[((int64_t)(t0 + base + tt) * Hv + h) * dv + cgrp * 32 + cc];
    }
    if (tid < cnt) {
      const int64_t tok = t0 + base + tid;
      sg[tid] = __expf(Lr.g[tok * Hv + h]);
      sb[tid] = Lr.beta[tok * Hv + h];
    }
    __syncthreads();
    for (int tt = 0; tt < cnt; ++tt) {
      const float decay = sg[tt];
      const float* kk = &sk[tt][rg];
      float kv = 0.f;
#pragma unroll
      for (int r = 0; r < 32; ++r) kv += S[r] * kk[4 * r];
      kv += __shfl_xor_sync(0xffffffffu, kv, 1);
      kv += __shfl_xor_sync(0xffffffffu, kv, 2);
      const float delta = sb[tt] * (sv[tt][c] - decay * kv);
#pragma unroll
      for (int r = 0; r < 32; ++r) S[r] = S[r] * decay + kk[4 * r] * delta;
    }
  }
  StateVec<ST>::store(Sp, S);
}

void gdn_spec_commit(torch::Tensor table, int64_t Hk, int64_t Hv, int64_t dv, int64_t C, int64_t W, int64_t ld,
                     bool state_f32, torch::Tensor seq_slot, torch::Tensor seq_start, torch::Tensor acc_len,
                     torch::Tensor seq_has_state) {
  const int64_t S = seq_slot.size(0), nl = table.size(0);
  if (S == 0 || nl == 0) return;
  TORCH_CHECK(table.is_cuda() && table.dtype() == torch::kInt64 && table.size(1) * 8 == (int64_t)sizeof(GdnCommitLayer),
              "gdn_spec_commit: layer table must be a device int64 [layers, 8] tensor");
  TORCH_CHECK(dv % 32 == 0 && W - 1 <= 8 && Hv % Hk == 0, "gdn_spec_commit: dv % 32, conv width <= 9");
  const at::cuda::CUDAGuard guard(seq_slot.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const dim3 grid((unsigned)S, (unsigned)(Hv * (dv / 32) + (C + 127) / 128), (unsigned)nl);
  const GdnCommitLayer* tab = reinterpret_cast<const GdnCommitLayer*>(table.data_ptr<int64_t>());
  if (state_f32)
    launch_pdl(gdn_spec_commit_kernel<float>, grid, dim3(128), 0, st, tab, (int)Hk, (int)Hv, (int)dv, (int)C,
               (int)W, ld, seq_slot.data_ptr<int32_t>(), seq_start.data_ptr<int32_t>(), acc_len.data_ptr<int32_t>(),
               seq_has_state.data_ptr<int32_t>());
  else
    launch_pdl(gdn_spec_commit_kernel<__nv_bfloat16>, grid, dim3(128), 0, st, tab, (int)Hk, (int)Hv, (int)dv,
               (int)C, (int)W, ld, seq_slot.data_ptr<int32_t>(), seq_start.data_ptr<int32_t>(),
               acc_len.data_ptr<int32_t>(), seq_has_state.data_ptr<int32_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k
