// Multi-head latent attention (MLA) with a lightning indexer and top-k sparse selection (GLM-5.3 /
// DeepSeek-V3.2 class, BASELINE configs 4 and 5), decode-oriented.
//
// Cache per attention layer: latent rows [blocks][64][576] bf16 = [rmsnorm(c_kv) (512) | rope(k_pe) (64)],
// and the indexer's keys [blocks][64][128] e4m3. Per query token t:
//   indexer : score[s] = sum_h w[t, h] * relu(q_i[t, h] . k_i[s])            (s < ctx(t))
//   top-k   : the k highest-scoring positions (all of them when ctx <= k), in position order
//   attention over the selected rows, heads absorbed into the latent space:
//             logit[h, s] = (q_lat[t, h] . c[s] + q_pe[t, h] . k_pe[s]) * scale,  o_lat[h] = softmax . c
//   then o[h] = W_uv[h] o_lat[h] (head_gemv) and the output projection.
// (reference: kernels/r9k_sparse_mla.hip:99-245 (split-K sparse MLA decode + combine),
// r9700_vllm/attn/indexer_logits.py (paged indexer logits, Triton there), r9700_vllm/models/glm5next.py:39-77
// (top_k_per_row).)
//
// Kernels: mla_cache_write (latent rmsnorm + rope + store, indexer key norm + rope + e4m3 store),
// rope_heads (rope of a strided head slice), indexer_score, topk_select (radix select, deterministic
// order), sparse_mla_decode (split over the selected rows, online softmax, 8 heads per CTA) +
// mla_combine, head_gemv (per-head [K -> N] projections: q absorption with W_uk, output with W_uv).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp8.h>
#include "common.cuh"

namespace r9k {

namespace {
constexpr int MLA_BLK = 64, LAT = 512, PE = 64, ROW = LAT + PE, IDXD = 128;

R9K_DEVINL float e4m3_to_f(uint8_t b) {
  __nv_fp8_e4m3 v;
  v.__x = b;
  return float(v);
}
R9K_DEVINL uint8_t f_to_e4m3(float f) {
  __nv_fp8_e4m3 v(fminf(fmaxf(f, -448.f), 448.f));
  return v.__x;
}
R9K_DEVINL int64_t slot_of(const int32_t* bt, int mb, int seq, int pos) {
  return (int64_t)bt[(int64_t)seq * mb + pos / MLA_BLK] * MLA_BLK + pos % MLA_BLK;
}
}  // namespace

R9K_DEVINL void cp_async16_sw(uint8_t* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// byte offset of 16-byte chunk c of row r in a 128-byte-swizzled tile (8-row groups of 1 KiB)
R9K_DEVINL uint32_t sw128_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// MN-major 128-byte-swizzled operand: rows along K (128 bytes = 64 elements of M or N per row), the two
// 64-element halves `lbo` bytes apart, 8-row groups `sbo` bytes apart
R9K_DEVINL uint64_t sdesc_mn_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// v[c] of every lane -> lane l returns the reduction of column l over the warp (transpose-reduce:
// each step trades the half of the columns this lane does not keep)
template <bool MAX>
R9K_DEVINL float col_reduce32(float (&v)[32], int lane) {
#pragma unroll
  for (int k = 16; k >= 1; k >>= 1) {
    const bool up = (lane & k) != 0;
#pragma unroll
    for (int i = 0; i < k; ++i) {
      const float send = up ? v[i] : v[i + k];
      const float recv = __shfl_xor_sync(0xffffffffu, send, k);
      const float keep = up ? v[i + k] : v[i];
      v[i] = MAX ? fmaxf(keep, recv) : keep + recv;
    }
  }
  return v[0];
}


// ------------------------------------------------------------------------------------------------
// cache write: one warp per token for the latent row, one for the indexer key
// ------------------------------------------------------------------------------------------------
__global__ void mla_cache_write_kernel(const __nv_bfloat16* __restrict__ kv, int64_t ldkv,
                                       const __nv_bfloat16* __restrict__ kv_w, const __nv_bfloat16* __restrict__ ik,
                                       int64_t ldik, const __nv_bfloat16* __restrict__ ik_w, float eps,
                                       const int32_t* __restrict__ positions, const float* __restrict__ cos_sin,
                                       const int32_t* __restrict__ slots, __nv_bfloat16* __restrict__ lat_cache,
                                       uint8_t* __restrict__ idx_cache, int T) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int t = warp >> 1, which = warp & 1;
  if (t >= T) return;
  const int64_t slot = slots[t];
  if (slot < 0) return;
  const int pos = positions[t];
  if (which == 0) {
    // latent: rmsnorm over 512 (16 per lane), then rope over the 64 pe dims (neox halves of 32)
    const __nv_bfloat16* src = kv + (int64_t)t * ldkv;
    float x[16];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      x[i] = __bfloat162float(src[lane + 32 * i]);
      ss += x[i] * x[i];
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rr = rsqrtf(ss / LAT + eps);
    __nv_bfloat16* dst = lat_cache + slot * ROW;
#pragma unroll
    for (int i = 0; i < 16; ++i) dst[lane + 32 * i] = __float2bfloat16(x[i] * rr * __bfloat162float(kv_w[lane + 32 * i]));
    const float* cs = cos_sin + (int64_t)pos * PE;
    const float a = __bfloat162float(src[LAT + lane]), b = __bfloat162float(src[LAT + 32 + lane]);
    const float c = cs[lane], s = cs[32 + lane];
    dst[LAT + lane] = __float2bfloat16(a * c - b * s);
    dst[LAT + 32 + lane] = __float2bfloat16(b * c + a * s);
  } else if (ik != nullptr) {
    // indexer key: rmsnorm over 128 (4 per lane), rope over the first 64 dims, e4m3
    const __nv_bfloat16* src = ik + (int64_t)t * ldik;
    float x[4];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[i] = __bfloat162float(src[lane + 32 * i]);
      ss += x[i] * x[i];
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rr = rsqrtf(ss / IDXD + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = x[i] * rr * __bfloat162float(ik_w[lane + 32 * i]);
    const float* cs = cos_sin + (int64_t)pos * PE;
    const float c = cs[lane], s = cs[32 + lane];
    const float a = x[0], b = x[1];  // dims lane and 32 + lane form the rotary pairs of the first 64
    x[0] = a * c - b * s;
    x[1] = b * c + a * s;
    uint8_t* dst = idx_cache + slot * IDXD;
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = f_to_e4m3(x[i]);
  }
}

// rope over dims [off, off + 64) of each head row: x [T, H, ld_h] (row stride ld_t), in place
__global__ void rope_heads_kernel(__nv_bfloat16* __restrict__ x, int64_t ld_t, int ld_h, int H, int off,
                                  const int32_t* __restrict__ positions, const float* __restrict__ cos_sin, int T) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T * H) return;
  const int t = warp / H, h = warp % H;
  __nv_bfloat16* p = x + (int64_t)t * ld_t + (int64_t)h * ld_h + off;
  const float* cs = cos_sin + (int64_t)positions[t] * PE;
  const float a = __bfloat162float(p[lane]), b = __bfloat162float(p[32 + lane]);
  const float c = cs[lane], s = cs[32 + lane];
  p[lane] = __float2bfloat16(a * c - b * s);
  p[32 + lane] = __float2bfloat16(b * c + a * s);
}

// ------------------------------------------------------------------------------------------------
// indexer scores: grid (T, ceil(max_ctx / 128)), one key per thread
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) indexer_score_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const float* __restrict__ w, int Hi,
    const uint8_t* __restrict__ idx_cache, const int32_t* __restrict__ bt, int mb, const int32_t* __restrict__ tok_seq,
    const int32_t* __restrict__ tok_ctx, float* __restrict__ scores, int64_t lds) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sq[];  // [Hi][128] then w [Hi]
  const int t = blockIdx.x, tid = threadIdx.x;
  const int ctx = tok_ctx[t], seq = tok_seq[t];
  const int s = blockIdx.y * 128 + tid;
  if ((int)blockIdx.y * 128 >= ctx) {
    if (s < lds) scores[(int64_t)t * lds + s] = -INFINITY;
    return;
  }
  float* sw = sq + Hi * IDXD;
  for (int e = tid; e < Hi * IDXD; e += 128) sq[e] = __bfloat162float(q[(int64_t)t * ldq + e]);
  for (int e = tid; e < Hi; e += 128) sw[e] = w[(int64_t)t * Hi + e];
  __syncthreads();
  if (s >= lds) return;
  if (s >= ctx) {
    scores[(int64_t)t * lds + s] = -INFINITY;
    return;
  }
  const uint8_t* kr = idx_cache + slot_of(bt, mb, seq, s) * IDXD;
  float k[IDXD];
#pragma unroll
  for (int i = 0; i < IDXD / 16; ++i) {
    const uint4 v = reinterpret_cast<const uint4*>(kr)[i];
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
#pragma unroll
    for (int j = 0; j < 16; ++j) k[16 * i + j] = e4m3_to_f(b[j]);
  }
  float acc = 0.f;
  for (int h = 0; h < Hi; ++h) {
    const float* qh = sq + h * IDXD;
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < IDXD; ++i) d = fmaf(qh[i], k[i], d);
    acc = fmaf(sw[h], fmaxf(d, 0.f), acc);
  }
  scores[(int64_t)t * lds + s] = acc;
}

// ------------------------------------------------------------------------------------------------
// top-k of each token's scores[0, ctx): radix select of the k-th largest key, then the selected
// positions in ascending order (greater-than first by position, ties filled lowest position first)
// ------------------------------------------------------------------------------------------------
R9K_DEVINL uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(1024) topk_select_kernel(const float* __restrict__ scores, int64_t lds,
                                                           const int32_t* __restrict__ tok_ctx, int k,
                                                           int32_t* __restrict__ out, int32_t* __restrict__ count) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_need;
  __shared__ uint32_t s_cnt[1024];
  const int t = blockIdx.x, tid = threadIdx.x;
  const int ctx = tok_ctx[t];
  const float* sc = scores + (int64_t)t * lds;
  int32_t* o = out + (int64_t)t * k;
  if (ctx <= k) {
    for (int i = tid; i < k; i += 1024) o[i] = i < ctx ? i : -1;
    if (tid == 0) count[t] = ctx;
    return;
  }
  if (tid == 0) {
    s_prefix = 0;
    s_need = (uint32_t)k;
  }
  // four 8-bit digit passes, most significant first
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += 1024) hist[i] = 0;
    __syncthreads();
    const uint32_t pre = s_prefix;
    const uint32_t mask = pass == 0 ? 0u : (0xFFFFFFFFu << (32 - 8 * pass));
    for (int i = tid; i < ctx; i += 1024) {
      const uint32_t key = order_key(sc[i]);
      if ((key & mask) == pre) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t need = s_need, acc = 0;
      int d = 255;
      for (; d > 0; --d) {
        if (acc + hist[d] >= need) break;
        acc += hist[d];
      }
      s_need = need - acc;
      s_prefix = pre | ((uint32_t)d << shift);
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;  // the k-th largest key; s_need of the keys equal to it are taken
  const uint32_t need_eq = s_need;
  // per-thread contiguous ranges keep the output in position order
  const int per = (ctx + 1023) / 1024;
  const int i0 = tid * per, i1 = min(ctx, i0 + per);
  uint32_t ngt = 0, neq = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = order_key(sc[i]);
    ngt += key > thr;
    neq += key == thr;
  }
  // exclusive scan of (ngt, neq) over threads, packed as 16 + 16 bits is too narrow; scan separately
  s_cnt[tid] = neq;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const uint32_t v = tid >= off ? s_cnt[tid - off] : 0u;
    __syncthreads();
    s_cnt[tid] += v;
    __syncthreads();
  }
  const uint32_t eq_before = s_cnt[tid] - neq;
  const uint32_t eq_take = eq_before >= need_eq ? 0u : min(neq, need_eq - eq_before);
  __syncthreads();
  s_cnt[tid] = ngt + eq_take;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const uint32_t v = tid >= off ? s_cnt[tid - off] : 0u;
    __syncthreads();
    s_cnt[tid] += v;
    __syncthreads();
  }
  uint32_t w = s_cnt[tid] - (ngt + eq_take);
  uint32_t eq_seen = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = order_key(sc[i]);
    if (key > thr) o[w++] = i;
    else if (key == thr && eq_seen < eq_take) {
      o[w++] = i;
      ++eq_seen;
    }
  }
  if (tid == 0) count[t] = k;
}

// ------------------------------------------------------------------------------------------------
// sparse MLA decode: grid (T, H / 8, nsplit), 256 threads; warp h <-> head (blockIdx.y * 8 + h)
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) sparse_mla_decode_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq_t, int ldq_h, int H, const __nv_bfloat16* __restrict__ lat_cache,
    const int32_t* __restrict__ bt, int mb, const int32_t* __restrict__ tok_seq, const int32_t* __restrict__ sel,
    const int32_t* __restrict__ sel_count, int k, float scale, int nsplit, float* __restrict__ part_o,
    float* __restrict__ part_ml) {
  pdl_wait();
  pdl_trigger();
  constexpr int HB = 8, KC = 32;
  __shared__ __align__(16) __nv_bfloat16 sqv[HB][ROW];
  __shared__ __align__(16) __nv_bfloat16 rows[KC][ROW];
  __shared__ float sp[HB][KC];
  __shared__ int sidx[KC];
  const int t = blockIdx.x, hb = blockIdx.y * HB, split = blockIdx.z, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int seq = tok_seq[t];
  const int n = sel_count[t];
  const int per = (n + nsplit - 1) / nsplit;
  const int j0 = split * per, j1 = min(n, j0 + per);
  for (int e = tid; e < HB * ROW; e += 256) {
    const int h = e / ROW, d = e % ROW;
    sqv[h][d] = (hb + h < H) ? q[(int64_t)t * ldq_t + (int64_t)(hb + h) * ldq_h + d] : __float2bfloat16(0.f);
  }
  float m = -INFINITY, l = 0.f, o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] = 0.f;
  for (int c0 = j0; c0 < j1; c0 += KC) {
    const int cnt = min(KC, j1 - c0);
    __syncthreads();
    if (tid < KC) sidx[tid] = tid < cnt ? sel[(int64_t)t * k + c0 + tid] : -1;
    __syncthreads();
    for (int e = tid; e < KC * (ROW / 8); e += 256) {
      const int r = e / (ROW / 8), c = e % (ROW / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (sidx[r] >= 0) v = reinterpret_cast<const uint4*>(lat_cache + slot_of(bt, mb, seq, sidx[r]) * ROW)[c];
      reinterpret_cast<uint4*>(&rows[r][0])[c] = v;
    }
    __syncthreads();
    // logits: warp = head, lane = row
    {
      float s = -INFINITY;
      if (lane < cnt && sidx[lane] >= 0) {
        float d = 0.f;
        const __nv_bfloat162* qh = reinterpret_cast<const __nv_bfloat162*>(sqv[warp]);
        const __nv_bfloat162* kr = reinterpret_cast<const __nv_bfloat162*>(rows[lane]);
#pragma unroll 8
        for (int i = 0; i < ROW / 2; ++i) {
          const float2 a = __bfloat1622float2(qh[i]), b = __bfloat1622float2(kr[i]);
          d = fmaf(a.x, b.x, fmaf(a.y, b.y, d));
        }
        s = d * scale;
      }
      float mx = s;
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m, mx);
      const float p = (s == -INFINITY) ? 0.f : __expf(s - m_new);
      float ps = p;
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      const float corr = (m == -INFINITY) ? 0.f : __expf(m - m_new);
      l = l * corr + ps;
      m = m_new;
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] *= corr;
      sp[warp][lane] = p;
    }
    __syncwarp();
    // o[h][lane * 16 + i] += sum_r p[h][r] * c[r][lane * 16 + i]
    for (int r = 0; r < cnt; ++r) {
      const float p = sp[warp][r];
      const __nv_bfloat16* cr = &rows[r][lane * 16];
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = fmaf(p, __bfloat162float(cr[i]), o[i]);
    }
  }
  const int h = hb + warp;
  if (h < H) {
    const int64_t base = ((int64_t)t * H + h) * nsplit + split;
    float* po = part_o + base * LAT + lane * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) po[i] = o[i];
    if (lane == 0) {
      part_ml[base * 2] = m;
      part_ml[base * 2 + 1] = l;
    }
  }
}

// o_lat[t, h, :] = sum_s exp(m_s - M) o_s / sum_s exp(m_s - M) l_s ; grid (T * H), 128 threads
__global__ void mla_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int nsplit,
                                   __nv_bfloat16* __restrict__ out, int64_t ldo_t, int ldo_h, int H) {
  pdl_wait();
  pdl_trigger();
  const int th = blockIdx.x, t = th / H, h = th % H, tid = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_ml[((int64_t)th * nsplit + s) * 2]);
  float L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < nsplit; ++s) {
    const float ms = part_ml[((int64_t)th * nsplit + s) * 2];
    if (ms == -INFINITY) continue;
    const float f = __expf(ms - M);
    L += f * part_ml[((int64_t)th * nsplit + s) * 2 + 1];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += f * part_o[((int64_t)th * nsplit + s) * LAT + tid + 128 * i];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) out[(int64_t)t * ldo_t + (int64_t)h * ldo_h + tid + 128 * i] = __float2bfloat16(acc[i] * inv);
}

// per-head projection: out[t, h, n] = sum_k x[t, h, k] W[h, n, k]; grid (H, ceil(N / 64), ceil(T / 16))
__global__ void __launch_bounds__(256) head_gemv_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx_t, int ldx_h,
                                                        const __nv_bfloat16* __restrict__ W, int N, int K,
                                                        __nv_bfloat16* __restrict__ out, int64_t ldo_t, int ldo_h, int T) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sx[];  // [16][K]
  const int h = blockIdx.x, n0 = blockIdx.y * 64, t0 = blockIdx.z * 16, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nt = min(16, T - t0);
  for (int e = tid; e < 16 * K; e += 256) {
    const int tt = e / K, kk = e % K;
    sx[e] = tt < nt ? __bfloat162float(x[(int64_t)(t0 + tt) * ldx_t + (int64_t)h * ldx_h + kk]) : 0.f;
  }
  __syncthreads();
  for (int nn = warp; nn < 64; nn += 8) {
    const int n = n0 + nn;
    if (n >= N) break;
    const __nv_bfloat16* wr = W + ((int64_t)h * N + n) * K;
    float acc[16];
#pragma unroll
    for (int tt = 0; tt < 16; ++tt) acc[tt] = 0.f;
    for (int kk = lane; kk < K; kk += 32) {
      const float wv = __bfloat162float(wr[kk]);
#pragma unroll
      for (int tt = 0; tt < 16; ++tt) acc[tt] = fmaf(wv, sx[tt * K + kk], acc[tt]);
    }
#pragma unroll
    for (int tt = 0; tt < 16; ++tt) {
      float v = acc[tt];
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0 && tt < nt) out[(int64_t)(t0 + tt) * ldo_t + (int64_t)h * ldo_h + n] = __float2bfloat16(v);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// host wrappers
// ------------------------------------------------------------------------------------------------
void mla_cache_write(torch::Tensor kv, torch::Tensor kv_w, c10::optional<torch::Tensor> ik,
                     c10::optional<torch::Tensor> ik_w, double eps, torch::Tensor positions, torch::Tensor cos_sin,
                     torch::Tensor slots, torch::Tensor lat_cache, c10::optional<torch::Tensor> idx_cache) {
  const int64_t T = kv.size(0);
  if (T == 0) return;
  TORCH_CHECK(kv.size(1) >= ROW && lat_cache.size(-1) == ROW && lat_cache.size(-2) == MLA_BLK, "mla_cache_write: shapes");
  TORCH_CHECK(cos_sin.size(1) == PE, "mla_cache_write: rope dim 64");
  const bool hi = ik.has_value() && ik->defined();
  const at::cuda::CUDAGuard guard(kv.device());
  auto bf = [](const torch::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); };
  const int64_t warps = 2 * T;
  launch_pdl(mla_cache_write_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0,
             at::cuda::getCurrentCUDAStream(), bf(kv), kv.stride(0), bf(kv_w), hi ? bf(*ik) : nullptr,
             hi ? ik->stride(0) : (int64_t)0, hi ? bf(*ik_w) : nullptr, (float)eps, positions.data_ptr<int32_t>(),
             cos_sin.data_ptr<float>(), slots.data_ptr<int32_t>(),
             reinterpret_cast<__nv_bfloat16*>(lat_cache.data_ptr()), hi ? idx_cache->data_ptr<uint8_t>() : nullptr,
             (int)T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_heads(torch::Tensor x, int64_t H, int64_t off, torch::Tensor positions, torch::Tensor cos_sin) {
  const int64_t T = x.size(0);
  if (T == 0) return;
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1 && cos_sin.size(1) == PE, "rope_heads: x [T, H, D]");
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t warps = T * H;
  launch_pdl(rope_heads_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0,
             at::cuda::getCurrentCUDAStream(), reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0),
             (int)x.stride(1), (int)H, (int)off, positions.data_ptr<int32_t>(), cos_sin.data_ptr<float>(), (int)T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------------------
// indexer scores on tcgen05: grid (T, ceil(max_ctx / 128)), 128 threads. Keys on the MMA's M side
// (128 positions per CTA, e4m3 rows widened to bf16 in shared memory: exact), the token's index heads
// on N, K = 128 dims: S^T [keys x heads] in TMEM; thread r (TMEM lane r) then sums w[h] relu(S[r][h])
// over its row, so the head reduction needs no cross-thread traffic.
// ------------------------------------------------------------------------------------------------
namespace sidx {
constexpr int KT = 128;
constexpr uint32_t KPLANE = KT * 128;                 // 64 dims of 128 keys, bf16
constexpr uint32_t OFF_K = 0, OFF_Q = 2 * KPLANE;     // then 2 planes of [HN rows][64 dims]
constexpr uint32_t QPLANE_MAX = 64 * 128;
constexpr int SMEM = (int)(OFF_Q + 2 * QPLANE_MAX) + 1024;
constexpr uint32_t TMEM_COLS = 64;
}  // namespace sidx

__global__ void __launch_bounds__(128) indexer_score_tc_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const float* __restrict__ w, int Hi, int HN,
    const uint8_t* __restrict__ idx_cache, const int32_t* __restrict__ bt, int mb, const int32_t* __restrict__ tok_seq,
    const int32_t* __restrict__ tok_ctx, float* __restrict__ scores, int64_t lds, int* __restrict__ status) {
  using namespace sidx;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_holder;
  __shared__ float sw[64];
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5;
  const uint32_t QPLANE = (uint32_t)HN * 128;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_holder;
  pdl_wait();
  pdl_trigger();
  const int ctx = tok_ctx[t], seq = tok_seq[t];
  const int s0 = blockIdx.y * KT, s = s0 + tid;
  if (s0 < ctx) {
    // the token's heads: 2 K-major planes of [HN rows][64 dims] (rows past Hi are zero)
    for (int e = tid; e < 2 * HN * 8; e += 128) {
      const int pl = e / (HN * 8), r = (e / 8) % HN, c = e % 8;
      uint8_t* dst = smem + OFF_Q + pl * QPLANE + sw128_off(r, c);
      if (r < Hi) cp_async16_sw(dst, q + (int64_t)t * ldq + r * IDXD + pl * 64 + c * 8);
      else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (tid < Hi) sw[tid] = w[(int64_t)t * Hi + tid];
    // key row tid: 128 e4m3 values widened to bf16 (exact) into the two K planes
    uint4 raw[8];
    if (s < ctx) {
      const uint4* kr = reinterpret_cast<const uint4*>(idx_cache + slot_of(bt, mb, seq, s) * IDXD);
#pragma unroll
      for (int i = 0; i < 8; ++i) raw[i] = kr[i];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) raw[i] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // 16 fp8 -> two 16-byte chunks of 8 bf16
      const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw[i]);
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf) {
        uint4 o;
        __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = __float2bfloat16(e4m3_to_f(b[hlf * 8 + j]));
        const int c16 = 2 * i + hlf;  // 16-byte chunk 0..15 of the 256-byte bf16 row
        *reinterpret_cast<uint4*>(smem + OFF_K + (c16 >> 3) * KPLANE + sw128_off(tid, c16 & 7)) = o;
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint32_t idesc = idesc_dense(kFmtBF16, kFmtBF16, 128, HN);
      const uint32_t kb = smem_u32(smem + OFF_K), qb = smem_u32(smem + OFF_Q);
#pragma unroll
      for (int pl = 0; pl < 2; ++pl)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tbase, sdesc_k_sw128(kb + pl * KPLANE + kk * 32), sdesc_k_sw128(qb + pl * QPLANE + kk * 32), idesc,
                     (pl | kk) ? 1u : 0u);
      tc_commit(&bar);
    }
    const bool ok = mbar_wait(&bar, 0, 1000000000ull);
    if (__syncthreads_and(ok)) {
      tc_fence_after();
      float acc = 0.f;
      const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < HN; c0 += 16) {
        float d[16];
        tmem_ld16(trow + c0, d);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < Hi) acc = fmaf(sw[c0 + j], fmaxf(d[j], 0.f), acc);
      }
      if (s < lds) scores[(int64_t)t * lds + s] = s < ctx ? acc : -INFINITY;
    } else {
      if (tid == 0) report_error(status, kErrMbarTimeout, 701, t);
      (void)mbar_wait(&bar, 0, 1000000000ull);
    }
  } else if (s < lds) {
    scores[(int64_t)t * lds + s] = -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

static bool indexer_tc_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("R9K_INDEXER");
    v = (e && (e[0] == 's')) ? 0 : 1;  // "simple" / "stock": the CUDA-core kernel
  }
  return v == 1;
}

void indexer_score(torch::Tensor q, torch::Tensor w, torch::Tensor idx_cache, torch::Tensor block_table,
                   torch::Tensor tok_seq, torch::Tensor tok_ctx, int64_t max_ctx, torch::Tensor scores,
                   c10::optional<torch::Tensor> status) {
  const int64_t T = q.size(0), Hi = q.size(1);
  if (T == 0) return;
  TORCH_CHECK(q.size(2) == IDXD && q.stride(2) == 1 && q.stride(1) == IDXD, "indexer_score: q [T, Hi, 128]");
  TORCH_CHECK(scores.size(1) >= max_ctx && Hi <= 64, "indexer_score: scores [T, >= max_ctx], <= 64 heads");
  const at::cuda::CUDAGuard guard(q.device());
  if (indexer_tc_enabled() && reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 && q.stride(0) % 8 == 0) {
    int* stt = (status.has_value() && status->defined()) ? status->data_ptr<int>() : nullptr;
    const int HN = (int)((Hi + 15) / 16 * 16);
    TORCH_CHECK(ensure_smem_attr((const void*)indexer_score_tc_kernel, sidx::SMEM) == cudaSuccess,
                "indexer_score: smem attribute");
    TORCH_CHECK(launch_pdl(indexer_score_tc_kernel, dim3((unsigned)T, (unsigned)((max_ctx + 127) / 128)), dim3(128),
                           (size_t)sidx::SMEM, at::cuda::getCurrentCUDAStream(),
                           reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0), w.data_ptr<float>(), (int)Hi,
                           HN, idx_cache.data_ptr<uint8_t>(), block_table.data_ptr<int32_t>(), (int)block_table.size(1),
                           tok_seq.data_ptr<int32_t>(), tok_ctx.data_ptr<int32_t>(), scores.data_ptr<float>(),
                           scores.stride(0), stt) == cudaSuccess,
                "indexer_score_tc launch");
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const size_t smem = (size_t)(Hi * IDXD + Hi) * sizeof(float);
  launch_pdl(indexer_score_kernel, dim3((unsigned)T, (unsigned)((max_ctx + 127) / 128)), dim3(128), smem,
             at::cuda::getCurrentCUDAStream(), reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0),
             w.data_ptr<float>(), (int)Hi, idx_cache.data_ptr<uint8_t>(), block_table.data_ptr<int32_t>(),
             (int)block_table.size(1), tok_seq.data_ptr<int32_t>(), tok_ctx.data_ptr<int32_t>(),
             scores.data_ptr<float>(), scores.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void topk_select(torch::Tensor scores, torch::Tensor tok_ctx, int64_t k, torch::Tensor out, torch::Tensor count) {
  const int64_t T = scores.size(0);
  if (T == 0) return;
  TORCH_CHECK(out.size(1) == k && out.dtype() == torch::kInt32, "topk_select: out [T, k] int32");
  const at::cuda::CUDAGuard guard(scores.device());
  launch_pdl(topk_select_kernel, dim3((unsigned)T), dim3(1024), 0, at::cuda::getCurrentCUDAStream(),
             scores.data_ptr<float>(), scores.stride(0), tok_ctx.data_ptr<int32_t>(), (int)k, out.data_ptr<int32_t>(),
             count.data_ptr<int32_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------------------
// sparse MLA on tcgen05: grid (T, ceil(H / 32), nsplit), 128 threads. The selected latent rows sit on
// the MMA's M side (128 keys per tile) and up to 32 heads on N:
//   S^T [keys x heads]  = K [keys x 576] . Q^T              (9 K-major planes of 64 dims each)
//   O^T [dims x heads] += V^T [dims x keys] . P^T [keys x heads]   (V^T: the same planes, MN-major)
// Thread r owns key row r (TMEM lane r) for the softmax; column (head) maxima and sums are butterfly
// reductions inside a warp (31 shuffles for 32 columns) and four partials across warps. O^T lives in
// TMEM (4 tiles of 128 dims x 32 heads) and is rescaled in place when a head's maximum grows. The
// gathered rows are written by cp.async into the 128-byte-swizzled layout the MMA descriptors read,
// so no tensor map (and no gather TMA) is involved. Partials (o, max, sum) go to mla_combine.
// (reference: kernels/r9k_sparse_mla.hip:99-205, the split-K sparse MLA decode it replaces with tensor
// cores; the math is the CUDA-core sparse_mla_decode_kernel above.)
// ------------------------------------------------------------------------------------------------
namespace smla {
constexpr int HN = 32, KT = 128, PLANES = ROW / 64;        // heads per CTA, keys per tile, 64-dim planes
constexpr uint32_t KPLANE = KT * 128, QPLANE = HN * 128;  // bytes
constexpr uint32_t OFF_K = 0, OFF_Q = OFF_K + PLANES * KPLANE, OFF_P = OFF_Q + PLANES * QPLANE;
constexpr uint32_t OFF_END = OFF_P + 2 * QPLANE;
constexpr int SMEM = (int)OFF_END + 1024;  // + 1 KiB alignment slack
constexpr uint32_t TMEM_COLS = 256, COL_S = 0, COL_O = 32;
}  // namespace smla

__global__ void __launch_bounds__(128, 1) sparse_mla_tc_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq_t, int ldq_h, int H, const __nv_bfloat16* __restrict__ lat_cache,
    const int32_t* __restrict__ bt, int mb, const int32_t* __restrict__ tok_seq, const int32_t* __restrict__ sel,
    const int32_t* __restrict__ sel_count, int k, float scale, int nsplit, float* __restrict__ part_o,
    float* __restrict__ part_ml, int* __restrict__ status) {
  using namespace smla;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_holder;
  __shared__ float red[4][32];
  __shared__ float s_mnew[32], s_corr[32];
  __shared__ int s_rescale;
  const int t = blockIdx.x, hb = blockIdx.y * HN, split = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint64_t timeout_ns = 1000000000ull;

  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_holder;
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);
  const uint32_t kbase = smem_u32(smem + OFF_K), qbase = smem_u32(smem + OFF_Q), pbase = smem_u32(smem + OFF_P);

  pdl_wait();  // queries, selections and the cache rows come from the preceding kernels
  pdl_trigger();
  const int seq = tok_seq[t];
  const int n = sel_count[t];
  const int per = (n + nsplit - 1) / nsplit;  // the CUDA-core kernel's partition of the selected rows
  const int j0 = min(n, split * per), j1 = min(n, j0 + per);

  // the CTA's heads as 9 K-major planes of [32 rows][64 dims]
  for (int e = tid; e < PLANES * HN * 8; e += 128) {
    const int pl = e / (HN * 8), r = (e / 8) % HN, c = e % 8;
    uint8_t* dst = smem + OFF_Q + pl * QPLANE + sw128_off(r, c);
    if (hb + r < H) cp_async16_sw(dst, q + (int64_t)t * ldq_t + (int64_t)(hb + r) * ldq_h + pl * 64 + c * 8);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");

  float m_run = -INFINITY, l_run = 0.f;  // running max / sum of head (hb + lane), kept by warp 0
  uint32_t phase = 0;
  int ntile = 0;
  bool failed = false;  // a bounded MMA wait ran out (uniform over the CTA)
  for (int c0 = j0; c0 < j1; c0 += KT) {
    const int cnt = min(KT, j1 - c0);
    const int pos = tid < cnt ? sel[(int64_t)t * k + c0 + tid] : -1;
    const bool live = pos >= 0;
    // key row tid -> row tid of every plane (zeros past the selection: V rows must stay finite)
    if (live) {
      const __nv_bfloat16* src = lat_cache + slot_of(bt, mb, seq, pos) * ROW;
#pragma unroll
      for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
        for (int c = 0; c < 8; ++c) cp_async16_sw(smem + OFF_K + pl * KPLANE + sw128_off(tid, c), src + pl * 64 + c * 8);
    } else {
#pragma unroll
      for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(smem + OFF_K + pl * KPLANE + sw128_off(tid, c)) = make_uint4(0, 0, 0, 0);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
    fence_proxy_async();  // generic-proxy shared writes -> the MMA's async-proxy reads
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      constexpr uint32_t idS = idesc_dense(kFmtBF16, kFmtBF16, 128, HN);
#pragma unroll 1
      for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tbase + COL_S, sdesc_k_sw128(kbase + pl * KPLANE + kk * 32),
                     sdesc_k_sw128(qbase + pl * QPLANE + kk * 32), idS, (pl | kk) ? 1u : 0u);
      tc_commit(&bar);
    }
    bool ok = mbar_wait(&bar, phase, timeout_ns);
    phase ^= 1;
    if (!__syncthreads_and(ok)) {
      failed = true;
      break;
    }
    tc_fence_after();
    float sv[32];
    tmem_ld16(trow + COL_S, sv);
    tmem_ld16(trow + COL_S + 16, sv + 16);
    tmem_ld_wait();
#pragma unroll
    for (int h = 0; h < 32; ++h) sv[h] = live ? sv[h] * scale : -INFINITY;
    {
      float v[32];
#pragma unroll
      for (int h = 0; h < 32; ++h) v[h] = sv[h];
      red[warp][lane] = col_reduce32<true>(v, lane);
    }
    __syncthreads();
    if (warp == 0) {
      const float mt = fmaxf(fmaxf(red[0][lane], red[1][lane]), fmaxf(red[2][lane], red[3][lane]));
      const float mn = fmaxf(m_run, mt);
      const float corr = (m_run == -INFINITY) ? 0.f : __expf(m_run - mn);
      s_mnew[lane] = mn;
      s_corr[lane] = corr;
      m_run = mn;
      const bool any = __any_sync(0xffffffffu, corr != 1.f);
      if (lane == 0) s_rescale = any ? 1 : 0;
    }
    __syncthreads();
    float pv[32];
#pragma unroll
    for (int h = 0; h < 32; ++h) {
      const float mn = s_mnew[h];
      const float e = (sv[h] == -INFINITY || mn == -INFINITY) ? 0.f : __expf(sv[h] - mn);
      pv[h] = __bfloat162float(__float2bfloat16(e));  // the sum counts what the MMA multiplies
    }
    {
      // P^T as the K-major B operand: [32 heads][128 keys] in two planes of 64 keys
      uint8_t* pl = smem + OFF_P + (tid >> 6) * QPLANE;
      const int kc = tid & 63, ch = kc >> 3, el = kc & 7;
#pragma unroll
      for (int h = 0; h < 32; ++h)
        *reinterpret_cast<__nv_bfloat16*>(pl + sw128_off(h, ch) + el * 2) = __float2bfloat16(pv[h]);
    }
    __syncthreads();
    red[warp][lane] = col_reduce32<false>(pv, lane);
    __syncthreads();
    if (warp == 0) l_run = l_run * s_corr[lane] + (red[0][lane] + red[1][lane] + red[2][lane] + red[3][lane]);
    if (ntile > 0 && s_rescale) {
      // O^T tile mt, lane = dim: scale head column h by corr[h]
#pragma unroll 1
      for (int mt = 0; mt < 4; ++mt) {
        float o[32];
        tmem_ld16(trow + COL_O + mt * HN, o);
        tmem_ld16(trow + COL_O + mt * HN + 16, o + 16);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 32; ++h) o[h] *= s_corr[h];
        tmem_st16(trow + COL_O + mt * HN, o);
        tmem_st16(trow + COL_O + mt * HN + 16, o + 16);
      }
      tmem_st_wait();
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      constexpr uint32_t idO = idesc_dense(kFmtBF16, kFmtBF16, 128, HN) | (1u << 15);  // A (V^T) MN-major
#pragma unroll 1
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_f16_ss(tbase + COL_O + mt * HN, sdesc_mn_sw128(kbase + 2 * mt * KPLANE + ks * 2048, KPLANE, 1024),
                     sdesc_k_sw128(pbase + (ks >> 2) * QPLANE + (ks & 3) * 32), idO, (ntile > 0 || ks > 0) ? 1u : 0u);
      tc_commit(&bar);
    }
    ok = mbar_wait(&bar, phase, timeout_ns);
    phase ^= 1;
    if (!__syncthreads_and(ok)) {
      failed = true;
      break;
    }
    tc_fence_after();
    ++ntile;
  }
  if (failed) {
    if (tid == 0) report_error(status, kErrMbarTimeout, 700, t);
    (void)mbar_wait(&bar, phase, timeout_ns);  // the last MMA batch, if it is still running
    ntile = 0;                                  // report an empty split
  }
  if (warp == 0 && hb + lane < H) {
    const int64_t base = ((int64_t)t * H + hb + lane) * nsplit + split;
    part_ml[base * 2] = ntile ? m_run : -INFINITY;
    part_ml[base * 2 + 1] = ntile ? l_run : 0.f;
  }
  const int hn = min(HN, H - hb);
#pragma unroll 1
  for (int mt = 0; mt < 4; ++mt) {
    float o[32];
    if (ntile) {
      tmem_ld16(trow + COL_O + mt * HN, o);
      tmem_ld16(trow + COL_O + mt * HN + 16, o + 16);
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int h = 0; h < 32; ++h) o[h] = 0.f;
    }
    const int d = mt * 128 + tid;
#pragma unroll
    for (int h = 0; h < 32; ++h)
      if (h < hn) part_o[(((int64_t)t * H + hb + h) * nsplit + split) * LAT + d] = o[h];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------
// sparse MLA on tcgen05, pipelined: the same math as sparse_mla_tc_kernel, with the phases of a tile
// overlapped across warps and with two CTAs per SM. Warp 0 gathers the selected rows into a ring of
// two slots, each holding two 64-dim planes of 128 keys (32 KiB); warp 1 issues the MMAs; warps 2-5
// run the softmax. Per 128-key tile the ring carries planes (0,1) (2,3) (4,5) (6,7) (8) for
// S^T = K Q^T, then (0,1) (2,3) (4,5) (6,7) again for O^T += V^T P^T (a re-read that the L2 serves),
// so the gather of the next planes runs under the MMAs and the softmax of the current ones. The
// softmax keeps the running max / sum of its 32 heads and rescales O^T in TMEM after the previous
// tile's P V has completed.
// ------------------------------------------------------------------------------------------------
namespace smla2 {
constexpr int HN = 32, KT = 128, PLANES = ROW / 64, NSLOT = 2, LOADS = 9;  // 5 S loads + 4 P V loads
constexpr uint32_t PLANE = KT * 128, SLOT = 2 * PLANE, QPLANE = HN * 128;
constexpr uint32_t OFF_Q = 0, OFF_RING = OFF_Q + PLANES * QPLANE, OFF_P = OFF_RING + NSLOT * SLOT;
constexpr uint32_t OFF_END = OFF_P + 2 * QPLANE;
constexpr int SMEM = (int)OFF_END + 1024;
constexpr uint32_t TMEM_COLS = 256, COL_S = 0, COL_O = 32;
constexpr uint64_t TIMEOUT = 1000000000ull;
}  // namespace smla2

R9K_DEVINL void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
R9K_DEVINL void named_bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// named barrier that also ORs a predicate over the participating threads (the same answer for all)
R9K_DEVINL bool named_bar_or(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(192, 2) sparse_mla_tc2_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq_t, int ldq_h, int H, const __nv_bfloat16* __restrict__ lat_cache,
    const int32_t* __restrict__ bt, int mb, const int32_t* __restrict__ tok_seq, const int32_t* __restrict__ sel,
    const int32_t* __restrict__ sel_count, int k, float scale, int nsplit, float* __restrict__ part_o,
    float* __restrict__ part_ml, int* __restrict__ status) {
  using namespace smla2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[NSLOT], empty[NSLOT], s_full, p_ready, pv_done, q_full;
  __shared__ uint32_t tmem_holder;
  __shared__ float red[4][32];
  __shared__ float s_mnew[32], s_corr[32];
  __shared__ int s_rescale;
  const int t = blockIdx.x, hb = blockIdx.y * HN, split = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&full[i], 32);  // one arrive per producer lane (cp.async completion, no increment)
      mbar_init(&empty[i], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&p_ready, 128);
    mbar_init(&pv_done, 1);
    mbar_init(&q_full, 32);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_holder;
  pdl_wait();
  pdl_trigger();
  const int seq = tok_seq[t];
  const int n = sel_count[t];
  const int per = (n + nsplit - 1) / nsplit;
  const int j0 = min(n, split * per), j1 = min(n, j0 + per);
  const int ntiles = (j1 - j0 + KT - 1) / KT;

  if (warp == 0) {
    // ------------------------------ gather producer ------------------------------
    // the CTA's heads as 9 K-major planes of [32 rows][64 dims]
    for (int e = lane; e < PLANES * HN * 8; e += 32) {
      const int pl = e / (HN * 8), r = (e / 8) % HN, c = e % 8;
      uint8_t* dst = smem + OFF_Q + pl * QPLANE + sw128_off(r, c);
      if (hb + r < H) cp_async16_sw(dst, q + (int64_t)t * ldq_t + (int64_t)(hb + r) * ldq_h + pl * 64 + c * 8);
      else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async();
    cp_async_mbar_arrive_noinc(&q_full);
    int load = 0;
    bool stop = false;
    for (int it = 0; it < ntiles && !stop; ++it) {
      const int c0 = j0 + it * KT, cnt = min(KT, j1 - c0);
      const __nv_bfloat16* src[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int r = lane + 32 * u;
        const int pos = r < cnt ? sel[(int64_t)t * k + c0 + r] : -1;
        src[u] = pos >= 0 ? lat_cache + slot_of(bt, mb, seq, pos) * ROW : nullptr;
      }
#pragma unroll 1
      for (int j = 0; j < LOADS; ++j, ++load) {
        const int sl = load % NSLOT;
        const bool got = mbar_wait(&empty[sl], (uint32_t)(((load / NSLOT) & 1) ^ 1), TIMEOUT);
        if (!__all_sync(0xffffffffu, got)) {
          if (lane == 0) report_error(status, kErrMbarTimeout, 702, load);
          stop = true;
          break;
        }
        const int p0 = j < 5 ? 2 * j : 2 * (j - 5);  // first plane of this load
        const int np = (j == 4) ? 1 : 2;             // load 4 carries plane 8 alone
        uint8_t* base = smem + OFF_RING + sl * SLOT;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int r = lane + 32 * u;
          for (int h = 0; h < np; ++h) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint8_t* dst = base + h * PLANE + sw128_off(r, c);
              if (src[u] != nullptr) cp_async16_sw(dst, src[u] + (p0 + h) * 64 + c * 8);
              else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
            }
          }
        }
        fence_proxy_async();
        cp_async_mbar_arrive_noinc(&full[sl]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idS = idesc_dense(kFmtBF16, kFmtBF16, 128, HN);
      constexpr uint32_t idO = idesc_dense(kFmtBF16, kFmtBF16, 128, HN) | (1u << 15);  // A (V^T) MN-major
      const uint32_t qbase = smem_u32(smem + OFF_Q), pbase = smem_u32(smem + OFF_P);
      bool ok = mbar_wait(&q_full, 0, TIMEOUT);
      int load = 0;
      for (int it = 0; it < ntiles && ok; ++it) {
        for (int j = 0; j < LOADS && ok; ++j, ++load) {
          const int sl = load % NSLOT;
          if (j == 5) {  // P of this tile written, O rescaled
            ok = mbar_wait(&p_ready, (uint32_t)(it & 1), TIMEOUT);
            if (!ok) break;
            tc_fence_after();
          }
          ok = mbar_wait(&full[sl], (uint32_t)((load / NSLOT) & 1), TIMEOUT);
          if (!ok) break;
          fence_proxy_async();
          tc_fence_after();
          const uint32_t sb = smem_u32(smem + OFF_RING + sl * SLOT);
          if (j < 5) {
            const int np = (j == 4) ? 1 : 2;
            for (int h = 0; h < np; ++h) {
              const int pl = 2 * j + h;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_f16_ss(tbase + COL_S, sdesc_k_sw128(sb + h * PLANE + kk * 32),
                           sdesc_k_sw128(qbase + pl * QPLANE + kk * 32), idS, (pl | kk) ? 1u : 0u);
            }
            tc_commit(&empty[sl]);
            if (j == 4) tc_commit(&s_full);
          } else {
            const int mt = j - 5;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              mma_f16_ss(tbase + COL_O + mt * HN, sdesc_mn_sw128(sb + ks * 2048, PLANE, 1024),
                         sdesc_k_sw128(pbase + (ks >> 2) * QPLANE + (ks & 3) * 32), idO,
                         (it > 0 || ks > 0) ? 1u : 0u);
            tc_commit(&empty[sl]);
            if (mt == 3) tc_commit(&pv_done);
          }
        }
      }
      if (!ok) report_error(status, kErrMbarTimeout, 703, load);
    }
    __syncwarp();
  } else {
    // ------------------------------ softmax (warps 2-5) ------------------------------
    // every control decision that could split the four warps goes through bar.red.or, so they all
    // take the same branch and meet at the same named barriers
    const int sw = warp - 2;                                    // 0..3 among the softmax warps
    const int row = (warp & 3) * 32 + lane;                     // TMEM lane this thread may access
    const uint32_t trow = tbase + ((uint32_t)((warp & 3) * 32) << 16);
    float m_run = -INFINITY, l_run = 0.f;  // head (hb + lane), kept by softmax warp 0
    bool fail = false;
    for (int it = 0; it < ntiles; ++it) {
      const int c0 = j0 + it * KT, cnt = min(KT, j1 - c0);
      const bool live = row < cnt && sel[(int64_t)t * k + c0 + row] >= 0;
      const bool bad = !mbar_wait(&s_full, (uint32_t)(it & 1), TIMEOUT);
      if (named_bar_or(1, 128, bad)) {
        fail = true;
        break;
      }
      tc_fence_after();
      float sv[32];
      tmem_ld16(trow + COL_S, sv);
      tmem_ld16(trow + COL_S + 16, sv + 16);
      tmem_ld_wait();
#pragma unroll
      for (int h = 0; h < 32; ++h) sv[h] = live ? sv[h] * scale : -INFINITY;
      {
        float v[32];
#pragma unroll
        for (int h = 0; h < 32; ++h) v[h] = sv[h];
        red[sw][lane] = col_reduce32<true>(v, lane);
      }
      named_bar_sync(1, 128);
      if (sw == 0) {
        const float mt = fmaxf(fmaxf(red[0][lane], red[1][lane]), fmaxf(red[2][lane], red[3][lane]));
        const float mn = fmaxf(m_run, mt);
        const float corr = (m_run == -INFINITY) ? 0.f : __expf(m_run - mn);
        s_mnew[lane] = mn;
        s_corr[lane] = corr;
        m_run = mn;
        const bool any = __any_sync(0xffffffffu, corr != 1.f);
        if (lane == 0) s_rescale = any ? 1 : 0;
      }
      named_bar_sync(1, 128);
      float pv[32];
#pragma unroll
      for (int h = 0; h < 32; ++h) {
        const float mn = s_mnew[h];
        const float e = (sv[h] == -INFINITY || mn == -INFINITY) ? 0.f : __expf(sv[h] - mn);
        pv[h] = __bfloat162float(__float2bfloat16(e));
      }
      // the previous tile's P V must be complete before P and O change
      const bool bad2 = it > 0 && !mbar_wait(&pv_done, (uint32_t)((it - 1) & 1), TIMEOUT);
      if (named_bar_or(1, 128, bad2)) {
        fail = true;
        break;
      }
      {
        uint8_t* pl = smem + OFF_P + (row >> 6) * QPLANE;
        const int kc = row & 63, ch = kc >> 3, el = kc & 7;
#pragma unroll
        for (int h = 0; h < 32; ++h)
          *reinterpret_cast<__nv_bfloat16*>(pl + sw128_off(h, ch) + el * 2) = __float2bfloat16(pv[h]);
      }
      red[sw][lane] = col_reduce32<false>(pv, lane);
      named_bar_sync(1, 128);
      if (sw == 0) l_run = l_run * s_corr[lane] + (red[0][lane] + red[1][lane] + red[2][lane] + red[3][lane]);
      if (it > 0 && s_rescale) {
        tc_fence_after();
#pragma unroll 1
        for (int mt = 0; mt < 4; ++mt) {
          float o[32];
          tmem_ld16(trow + COL_O + mt * HN, o);
          tmem_ld16(trow + COL_O + mt * HN + 16, o + 16);
          tmem_ld_wait();
#pragma unroll
          for (int h = 0; h < 32; ++h) o[h] *= s_corr[h];
          tmem_st16(trow + COL_O + mt * HN, o);
          tmem_st16(trow + COL_O + mt * HN + 16, o + 16);
        }
        tmem_st_wait();
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&p_ready);
      named_bar_sync(1, 128);  // red[] and s_* are rewritten by the next tile
    }
    // epilogue: after the last tile's P V
    if (ntiles > 0 && !fail) {
      const bool bad = !mbar_wait(&pv_done, (uint32_t)((ntiles - 1) & 1), TIMEOUT);
      fail = named_bar_or(1, 128, bad);
    }
    const bool done = ntiles > 0 && !fail;
    if (fail && sw == 0 && lane == 0) report_error(status, kErrMbarTimeout, 704, t);
    tc_fence_after();
    if (sw == 0 && hb + lane < H) {
      const int64_t base = ((int64_t)t * H + hb + lane) * nsplit + split;
      part_ml[base * 2] = done ? m_run : -INFINITY;
      part_ml[base * 2 + 1] = done ? l_run : 0.f;
    }
    const int hn = min(HN, H - hb);
#pragma unroll 1
    for (int mt = 0; mt < 4; ++mt) {
      float o[32];
      if (done) {
        tmem_ld16(trow + COL_O + mt * HN, o);
        tmem_ld16(trow + COL_O + mt * HN + 16, o + 16);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int h = 0; h < 32; ++h) o[h] = 0.f;
      }
      const int d = mt * 128 + row;
#pragma unroll
      for (int h = 0; h < 32; ++h)
        if (h < hn) part_o[(((int64_t)t * H + hb + h) * nsplit + split) * LAT + d] = o[h];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

// 1: single-stage kernel always (R9K_MLA_ATTN=tc1); 0: by grid size (the pipelined kernel needs two
// CTAs on every SM to pay for its re-read of the V planes: measured 2.51 vs 2.75 ms at 1024 tokens x 64
// heads x top-2048, 58 vs 48 us at 16 tokens)
static int mla_tc_mode() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("R9K_MLA_ATTN");
    v = (e && strcmp(e, "tc1") == 0) ? 1 : 0;
  }
  return v;
}

void sparse_mla_decode_tc(torch::Tensor q, torch::Tensor lat_cache, torch::Tensor block_table, torch::Tensor tok_seq,
                          torch::Tensor sel, torch::Tensor sel_count, double scale, torch::Tensor part_o,
                          torch::Tensor part_ml, torch::Tensor out, torch::Tensor status) {
  const int64_t T = q.size(0), H = q.size(1);
  if (T == 0) return;
  TORCH_CHECK(q.dtype() == torch::kBFloat16 && q.size(2) >= ROW && q.stride(2) == 1 && q.stride(1) % 8 == 0 &&
                  q.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0,
              "sparse_mla_decode_tc: q [T, H, 576] bf16 with 16-byte aligned rows");
  TORCH_CHECK(lat_cache.dtype() == torch::kBFloat16 && lat_cache.is_contiguous() && lat_cache.size(-1) == ROW,
              "sparse_mla_decode_tc: latent cache [blocks, 64, 576] bf16");
  const int64_t nsplit = part_o.size(1);
  TORCH_CHECK(part_o.size(0) >= T * H && part_o.size(2) == LAT && part_o.is_contiguous() && part_ml.is_contiguous(),
              "sparse_mla_decode_tc: partials [T*H, nsplit, 512]");
  TORCH_CHECK(T <= 2147483647 && nsplit <= 65535, "sparse_mla_decode_tc: grid");
  const at::cuda::CUDAGuard guard(q.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int64_t ctas = T * ((H + smla::HN - 1) / smla::HN) * nsplit;
  const bool v2 = mla_tc_mode() == 0 && ctas >= 2 * device_sm_count();
  auto kern = v2 ? sparse_mla_tc2_kernel : sparse_mla_tc_kernel;
  const int smem = v2 ? smla2::SMEM : smla::SMEM;
  TORCH_CHECK(ensure_smem_attr((const void*)kern, smem) == cudaSuccess, "sparse_mla_decode_tc: smem attribute");
  TORCH_CHECK(launch_pdl(kern, dim3((unsigned)T, (unsigned)((H + smla::HN - 1) / smla::HN), (unsigned)nsplit),
                         dim3(v2 ? 192 : 128), (size_t)smem, st, reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()),
                         q.stride(0), (int)q.stride(1), (int)H,
                         reinterpret_cast<const __nv_bfloat16*>(lat_cache.data_ptr()), block_table.data_ptr<int32_t>(),
                         (int)block_table.size(1), tok_seq.data_ptr<int32_t>(), sel.data_ptr<int32_t>(),
                         sel_count.data_ptr<int32_t>(), (int)sel.size(1), (float)scale, (int)nsplit,
                         part_o.data_ptr<float>(), part_ml.data_ptr<float>(), status.data_ptr<int>()) == cudaSuccess,
              "sparse_mla_decode_tc launch");
  launch_pdl(mla_combine_kernel, dim3((unsigned)(T * H)), dim3(128), 0, st, part_o.data_ptr<float>(),
             part_ml.data_ptr<float>(), (int)nsplit, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0),
             (int)out.stride(1), (int)H);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sparse_mla_decode(torch::Tensor q, torch::Tensor lat_cache, torch::Tensor block_table, torch::Tensor tok_seq,
                       torch::Tensor sel, torch::Tensor sel_count, double scale, torch::Tensor part_o,
                       torch::Tensor part_ml, torch::Tensor out) {
  const int64_t T = q.size(0), H = q.size(1);
  if (T == 0) return;
  TORCH_CHECK(q.size(2) >= ROW && q.stride(2) == 1, "sparse_mla_decode: q [T, H, 576] (latent | rope)");
  const int64_t nsplit = part_o.size(1);
  TORCH_CHECK(part_o.size(0) >= T * H && part_o.size(2) == LAT && part_o.is_contiguous() && part_ml.is_contiguous(),
              "sparse_mla_decode: partials [T*H, nsplit, 512]");
  const at::cuda::CUDAGuard guard(q.device());
  auto st = at::cuda::getCurrentCUDAStream();
  launch_pdl(sparse_mla_decode_kernel, dim3((unsigned)T, (unsigned)((H + 7) / 8), (unsigned)nsplit), dim3(256), 0, st,
             reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0), (int)q.stride(1), (int)H,
             reinterpret_cast<const __nv_bfloat16*>(lat_cache.data_ptr()), block_table.data_ptr<int32_t>(),
             (int)block_table.size(1), tok_seq.data_ptr<int32_t>(), sel.data_ptr<int32_t>(),
             sel_count.data_ptr<int32_t>(), (int)sel.size(1), (float)scale, (int)nsplit, part_o.data_ptr<float>(),
             part_ml.data_ptr<float>());
  launch_pdl(mla_combine_kernel, dim3((unsigned)(T * H)), dim3(128), 0, st, part_o.data_ptr<float>(),
             part_ml.data_ptr<float>(), (int)nsplit, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0),
             (int)out.stride(1), (int)H);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void head_gemv(torch::Tensor x, torch::Tensor W, torch::Tensor out) {
  const int64_t T = x.size(0), H = W.size(0), N = W.size(1), K = W.size(2);
  if (T == 0) return;
  TORCH_CHECK(x.size(1) == H && x.size(2) == K && x.stride(2) == 1 && W.is_contiguous() && out.stride(2) == 1,
              "head_gemv: x [T, H, K], W [H, N, K], out [T, H, N]");
  const at::cuda::CUDAGuard guard(x.device());
  const size_t smem = 16 * K * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "head_gemv: K too large");
  cudaFuncSetAttribute(head_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_pdl(head_gemv_kernel, dim3((unsigned)H, (unsigned)((N + 63) / 64), (unsigned)((T + 15) / 16)), dim3(256), smem,
             at::cuda::getCurrentCUDAStream(), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
             (int)x.stride(1), reinterpret_cast<const __nv_bfloat16*>(W.data_ptr()), (int)N, (int)K,
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), (int)out.stride(1), (int)T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k
