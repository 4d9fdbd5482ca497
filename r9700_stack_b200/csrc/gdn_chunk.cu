// Chunked gated delta rule for prefill on tcgen05 (sm_100a).
//
// The token-serial recurrence (gdn.cu) does ~6 FLOP per state element per token on CUDA cores with a
// shuffle reduction on the critical path of every token. For long prompts the same result is computed
// chunk-wise (the WY / UT form of the delta rule; the reference keeps this form for long prefill in
// its stock chunked core, r9700_vllm/models/gdn.py:28-33). Per sequence, value head h and chunk of
// C = 128 tokens with cumulative log-decay gc_t (gamma_t = exp(gc_t)), state S (dk x dv) entering the
// chunk:
//   L[t][j] = beta_t exp(gc_t - gc_j) k_t . k_j   (j < t)        T = (I + L)^-1   (unit lower)
//   P[t][j] = exp(gc_t - gc_j) q_t . k_j          (j <= t)
//   U = T (beta v),   W = T (beta gamma k)                          (chunk-local, no S)
//   Delta = U - W S,  O = (gamma q) S + P Delta,  S' = gamma_C S + (gamma_C / gamma k)^T Delta
// Phase 1 (gdn_chunk_prep, one CTA per chunk and value head, all in parallel): KK^T and QK^T on the
// tensor cores, the masks and decays, T by blocked forward substitution in fp32, then U and W on the
// tensor cores (V and K enter as MN-major operands in their natural row layout). It writes the
// operands of phase 2 (bf16 W, gamma q, K-hat and P rows; fp32 U^T).
// Phase 2 (gdn_chunk_scan, one CTA per sequence and value head, chunks in order): everything is kept
// transposed so TMEM lane n is state column n (dv): the state S^T lives in TMEM in fp32 for the whole
// sequence; per chunk
//   MMA1  Delta^T_acc = S^T W^T        MMA2  O^T = S^T (gamma q)^T
//   E1    Delta^T = U^T - Delta^T_acc (bf16 operand), S^T *= gamma_C (in TMEM)
//   MMA3  S^T += Delta^T K-hat (MN-major) MMA4  O^T += Delta^T P^T
//   E2    O^T -> o (fp32, the same layout gdn_recurrent writes), S^T -> bf16 operand of the next MMA1
// The operand tiles of the next chunk stream in by TMA while the current chunk's epilogues run.
// All MMAs are kind::f16 with bf16 operands and fp32 accumulation, M = N = 128, K = 128 (8 steps).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "tmap.h"

namespace r9k {
namespace gch {
constexpr int C = 128;              // tokens per chunk
constexpr int D = 128;              // head dim (dk == dv)
constexpr int REG = 128 * 128;      // one 128-row x 64-element bf16 swizzle region (16 KB)
constexpr int TILE = 2 * REG;       // a 128 x 128 bf16 operand (two regions along K)
constexpr int LS = 129;             // fp32 row stride of L / T in shared memory (bank spread)
// phase 1 shared memory (operand tiles 1 KB aligned for the 128-byte swizzle)
constexpr int P1_Q = 0;             // q rows (TMA; A of QK^T), then T diag(beta) (A of U)
constexpr int P1_K = TILE;          // k rows (TMA; A and B of KK^T, MN-major B of W)
constexpr int P1_V = 2 * TILE;      // v rows (TMA; MN-major B of U)
constexpr int P1_T2 = 3 * TILE;     // T diag(beta gamma) (A of W)
constexpr int P1_L = 4 * TILE;      // L fp32 [128][LS], turned into T in place
constexpr int P1_X = P1_L + C * LS * 4;  // off-diagonal products of the blocked solve [16][LS]
constexpr int P1_BAR = P1_X + 16 * LS * 4;
constexpr int P1_SMEM = P1_BAR + 64 + 1024;
// phase 2 shared memory
constexpr int P2_S = 0, P2_D = TILE, P2_W = 2 * TILE, P2_Q = 3 * TILE, P2_K = 4 * TILE, P2_P = 5 * TILE;
constexpr int P2_BAR = 6 * TILE;
constexpr int P2_SMEM = P2_BAR + 128 + 1024;
}  // namespace gch

R9K_DEVINL float to_float(float x) { return x; }
R9K_DEVINL float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> R9K_DEVINL T from_float(float x);
template <> R9K_DEVINL float from_float<float>(float x) { return x; }
template <> R9K_DEVINL __nv_bfloat16 from_float<__nv_bfloat16>(float x) { return __float2bfloat16(x); }

// 8 floats -> 8 bf16 in one 16-byte word
R9K_DEVINL uint4 pack8_bf16(const float* x) {
  uint4 r;
  __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
  r.x = *reinterpret_cast<uint32_t*>(&h[0]);
  r.y = *reinterpret_cast<uint32_t*>(&h[1]);
  r.z = *reinterpret_cast<uint32_t*>(&h[2]);
  r.w = *reinterpret_cast<uint32_t*>(&h[3]);
  return r;
}
// 16 consecutive elements [e0, e0 + 16) of row r of a 128x128 bf16 K-major operand (128-byte swizzle)
R9K_DEVINL void st_tile16(uint8_t* tile, int r, int e0, const float* x) {
  uint8_t* reg = tile + (e0 >> 6) * gch::REG;
  const int c0 = (e0 & 63) >> 3;
#pragma unroll
  for (int i = 0; i < 2; ++i)
    *reinterpret_cast<uint4*>(reg + r * 128 + (((c0 + i) ^ (r & 7)) << 4)) = pack8_bf16(x + 8 * i);
}
// 128x128x128 bf16 MMA, both operands K-major 128-byte-swizzled tiles: d (+)= a b^T
R9K_DEVINL void mma_tile(uint32_t d, uint32_t a, uint32_t b, uint32_t accumulate) {
  constexpr uint32_t idesc = idesc_dense(kFmtBF16, kFmtBF16, 128, 128);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t off = (uint32_t)((k >> 2) * gch::REG + (k & 3) * 32);
    mma_f16_ss(d, sdesc_k_sw128(a + off), sdesc_k_sw128(b + off), idesc, (accumulate || k > 0) ? 1u : 0u);
  }
}

// 128-byte-swizzled MN-major operand: rows along K (128 bytes = 64 bf16 of N per row), the two N-halves
// `lbo` bytes apart, 8-row groups `sbo` bytes apart
R9K_DEVINL uint64_t sdesc_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}
// d (+)= a b with a K-major [M rows][K] and b MN-major [K rows][N] (rows of 128 bf16 in two regions)
R9K_DEVINL void mma_tile_mn(uint32_t d, uint32_t a, uint32_t b, uint32_t accumulate) {
  constexpr uint32_t idesc = idesc_dense(kFmtBF16, kFmtBF16, 128, 128) | (1u << 16);  // B MN-major
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t aoff = (uint32_t)((k >> 2) * gch::REG + (k & 3) * 32);
    mma_f16_ss(d, sdesc_k_sw128(a + aoff), sdesc_mn(b + (uint32_t)(k * 16 * 128), gch::REG, 1024), idesc,
               (accumulate || k > 0) ? 1u : 0u);
  }
}
// 16 consecutive elements [e0, e0 + 16) of row r of a swizzled bf16 tile, as floats
R9K_DEVINL void ld_tile16(const uint8_t* tile, int r, int e0, float* x) {
  const uint8_t* reg = tile + (e0 >> 6) * gch::REG;
  const int c0 = (e0 & 63) >> 3;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint4 v = *reinterpret_cast<const uint4*>(reg + r * 128 + (((c0 + i) ^ (r & 7)) << 4));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      x[8 * i + 2 * j] = f.x;
      x[8 * i + 2 * j + 1] = f.y;
    }
  }
}

struct ChunkArgs {
  const float* g;      // [T, Hv] log decay
  const float* beta;   // [T, Hv]
  int Hk, Hv;
  const int32_t* ctab;  // [chunks][3]: first token, tokens (1..128), sequence row
  int nchunks;
  // phase 1 outputs / phase 2 operands, per (chunk, head) at index (chunk * Hv + head)
  __nv_bfloat16* w;    // [.., 128 tokens, 128 dk]
  __nv_bfloat16* qg;   // gamma q [.., 128 tokens, 128 dk]
  __nv_bfloat16* kh;   // gamma_C / gamma k [.., 128 tokens, 128 dk]
  __nv_bfloat16* p;    // [.., 128 t, 128 j]
  float* uT;           // U^T [.., 128 dv, 128 tokens]
  float* gC;           // gamma_C [..]
  // phase 2
  const int32_t* seq_chunk0;  // [S + 1]: chunk range of each sequence
  const int32_t* seq_slot;
  const int32_t* seq_has_state;
  int write_state;
  float* o;            // [T, Hv, 128]
  int* status;
  uint64_t timeout_ns;
  unsigned long long* trace;  // tuning: 8 %globaltimer stamps per phase-1 CTA, or null
};

// ------------------------------------------------------------------------------------------------
// Phase 1: grid (chunks, Hv), 256 threads (token row t = tid % 128, each half of the threads taking half of
// a row's columns; the blocked solve spreads over all 256). q, k, v arrive as bf16 tiles by TMA
// from the conv step's [T, 2 Hk + Hv, 128] copy (one round trip); every later operand is formed in
// shared memory or TMEM, so nothing is gathered column-wise from global memory.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 1) gdn_chunk_prep_kernel(const __grid_constant__ CUtensorMap tmQKV,
                                                                const ChunkArgs a) {
  using namespace gch;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Qt = smem + P1_Q;
  uint8_t* Kt = smem + P1_K;
  uint8_t* Vt = smem + P1_V;
  uint8_t* T2 = smem + P1_T2;
  float* Ls = reinterpret_cast<float*>(smem + P1_L);  // L, then T (in place)
  float* Xs = reinterpret_cast<float*>(smem + P1_X);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + P1_BAR);  // [0] tiles landed, [1] MMA done
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + P1_BAR + 32);
  __shared__ float sgc[C], sb[C], sgam[C];
  __shared__ float swsum[4];
  const int cid = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = a.ctab[3 * cid], n = a.ctab[3 * cid + 1];
  const int kh = h / (a.Hv / a.Hk);
  const int64_t oidx = (int64_t)cid * a.Hv + h;
  unsigned long long* tr = (a.trace != nullptr && tid == 0) ? a.trace + oidx * 8 : nullptr;
  if (tr) tr[0] = globaltimer_ns();
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    prefetch_tmap(&tmQKV);
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *tmem_holder;
  pdl_wait();
  if (tid == 0) {
    // rows t0 .. t0 + 127 of head columns (q: kh, k: Hk + kh, v: 2 Hk + h); rows past the step's tokens
    // read zeros, rows of the next sequence are masked below
    mbar_arrive_expect_tx(&bar[0], 3 * TILE);
    const int heads[3] = {kh, a.Hk + kh, 2 * a.Hk + h};
    uint8_t* dst[3] = {Qt, Kt, Vt};
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      tma_load_3d_hint(dst[i], &tmQKV, &bar[0], 0, heads[i], t0, policy_evict_first());
      tma_load_3d_hint(dst[i] + REG, &tmQKV, &bar[0], 64, heads[i], t0, policy_evict_first());
    }
  }
  // gates: inclusive prefix sum of the log decay over the chunk (warp scans + warp offsets)
  {
    const int t = tid & 127;
    float sacc = 0.f;
    if (tid < 128) {
      const float gv = t < n ? a.g[(int64_t)(t0 + t) * a.Hv + h] : 0.f;
      sb[t] = t < n ? a.beta[(int64_t)(t0 + t) * a.Hv + h] : 0.f;
      sacc = gv;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, sacc, o);
        if (lane >= o) sacc += y;
      }
      if (lane == 31) swsum[warp] = sacc;
    }
    __syncthreads();
    if (tid < 128) {
      for (int w = 0; w < warp; ++w) sacc += swsum[w];
      sgc[t] = sacc;
      sgam[t] = __expf(sacc);
    }
  }
  __syncthreads();
  const bool ok0 = mbar_wait(&bar[0], 0, a.timeout_ns);
  if (!ok0) report_error(a.status, kErrMbarTimeout, 600, 0);
  if (tr) tr[1] = globaltimer_ns();
  if (tid == 0 && ok0) {
    tc_fence_after();
    mma_tile(tb, smem_u32(Kt), smem_u32(Kt), 0);        // KK^T -> cols [0, 128)
    mma_tile(tb + 128, smem_u32(Qt), smem_u32(Kt), 0);  // QK^T -> cols [128, 256)
    tc_commit(&bar[1]);
  }
  // while the tensor cores run: gamma q rows and K-hat rows (gamma_C / gamma_t k_t) to global
  const float gcl = sgc[n - 1];
  const int half = tid >> 7;  // 256 threads: token row t = tid % 128, column half `half`
  {
    const int t = tid & 127;
    const bool in = t < n;
    const float gq = in ? sgam[t] : 0.f, gk = in ? __expf(fminf(gcl - sgc[t], 0.f)) : 0.f;
    __nv_bfloat16* qd = a.qg + (oidx * C + t) * D;
    __nv_bfloat16* kd = a.kh + (oidx * C + t) * D;
#pragma unroll 1
    for (int e = half * 64; e < half * 64 + 64; e += 16) {
      float x[16], y[16];
      ld_tile16(Qt, t, e, x);
      ld_tile16(Kt, t, e, y);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        x[i] *= gq;
        y[i] *= gk;
      }
      *reinterpret_cast<uint4*>(qd + e) = pack8_bf16(x);
      *reinterpret_cast<uint4*>(qd + e + 8) = pack8_bf16(x + 8);
      *reinterpret_cast<uint4*>(kd + e) = pack8_bf16(y);
      *reinterpret_cast<uint4*>(kd + e + 8) = pack8_bf16(y + 8);
    }
  }
  const bool ok1 = ok0 && __syncthreads_and(mbar_wait(&bar[1], 0, a.timeout_ns));
  if (!ok1 && tid == 0) report_error(a.status, kErrMbarTimeout, 601, 0);
  if (tr) tr[2] = globaltimer_ns();
  tc_fence_after();
  const uint32_t trow = tb + ((uint32_t)((warp & 3) * 32) << 16);  // warps w and w + 4 share a lane quadrant
  // ---- L row t (shared, fp32) and P row t (global, bf16)
  {
    const int t = tid & 127;
    const float gct = sgc[t], bt = sb[t];
    __nv_bfloat16* pd = a.p + (oidx * C + t) * C;
#pragma unroll 1
    for (int j0 = half * 64; j0 < half * 64 + 64; j0 += 16) {
      float kk[16], qk[16];
      if (ok1) {
        tmem_ld16(trow + j0, kk);
        tmem_ld16(trow + 128 + j0, qk);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) kk[i] = qk[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = j0 + i;
        const float dec = __expf(fminf(gct - sgc[j], 0.f));
        Ls[t * LS + j] = (j < t && t < n) ? bt * dec * kk[i] : 0.f;
        qk[i] = (j <= t && t < n) ? dec * qk[i] : 0.f;
      }
      *reinterpret_cast<uint4*>(pd + j0) = pack8_bf16(qk);
      *reinterpret_cast<uint4*>(pd + j0 + 8) = pack8_bf16(qk + 8);
    }
  }
  __syncthreads();
  if (tr) tr[3] = globaltimer_ns();
  // ---- T = (I + L)^-1 in place, blocks of 16 rows: diagonal blocks by forward substitution (thread =
  // column of its block), then block row i: X = L[i, <i] T[<i, <i], T[i, <i] = -T_ii X
  {
    const int bi = (tid >> 4) & 7, cc = tid & 15, base = bi * 16;
    float tcol[16];
    if (tid < 128) {
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < r; ++j) acc += Ls[(base + r) * LS + base + j] * tcol[j];
        tcol[r] = r < cc ? 0.f : (r == cc ? 1.f : -acc);
      }
    }
    __syncthreads();  // every thread has read its diagonal block of L
    if (tid < 128) {
#pragma unroll
      for (int r = 0; r < 16; ++r) Ls[(base + r) * LS + base + cc] = tcol[r];
      for (int c2 = base + 16; c2 < C; ++c2) Ls[(base + cc) * LS + c2] = 0.f;  // strictly upper blocks
    }
  }
  __syncthreads();
#pragma unroll 1
  for (int i = 1; i < 8; ++i) {
    const int r = tid & 15, cg = tid >> 4;
    const int row = (16 * i + r) * LS;
    // thread (r, cg) owns X[r][cg + 16 m], m < i: one L load per k2 feeds all of its columns
    // (independent accumulators, loads of T broadcast across the 16 threads of a column group)
    float acc[7];
#pragma unroll
    for (int m = 0; m < 7; ++m) acc[m] = 0.f;
#pragma unroll 2
    for (int k2 = 0; k2 < 16 * i; ++k2) {
      const float lv = Ls[row + k2];
#pragma unroll
      for (int m = 0; m < 7; ++m) {
        const int c = cg + 16 * m;
        if (m < i && k2 >= c) acc[m] += lv * Ls[k2 * LS + c];
      }
    }
#pragma unroll
    for (int m = 0; m < 7; ++m)
      if (m < i) Xs[r * LS + cg + 16 * m] = acc[m];
    __syncthreads();
    for (int c = cg; c < 16 * i; c += 16) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) acc += Ls[row + 16 * i + m] * Xs[m * LS + c];
      Ls[row + c] = -acc;  // L[i, <i] is consumed (in X); T_ii[r][m] is zero for m > r
    }
    __syncthreads();
  }
  if (tr) tr[4] = globaltimer_ns();
  // ---- T diag(beta) (A of U, over the q tile) and T diag(beta gamma) (A of W)
  {
    const int t = tid & 127;
#pragma unroll 1
    for (int e = half * 64; e < half * 64 + 64; e += 16) {
      float x[16], y[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float tv = Ls[t * LS + e + i];
        x[i] = tv * sb[e + i];
        y[i] = tv * sb[e + i] * sgam[e + i];
      }
      st_tile16(Qt, t, e, x);
      st_tile16(T2, t, e, y);
    }
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0 && ok1) {
    mma_tile_mn(tb, smem_u32(Qt), smem_u32(Vt), 0);        // U = T diag(beta) V          -> cols [0, 128)
    mma_tile_mn(tb + 128, smem_u32(T2), smem_u32(Kt), 0);  // W = T diag(beta gamma) K    -> cols [128, 256)
    tc_commit(&bar[1]);
  }
  if (tr) tr[5] = globaltimer_ns();
  const bool ok2 = ok1 && __syncthreads_and(mbar_wait(&bar[1], 1, a.timeout_ns));
  if (!ok2 && tid == 0) report_error(a.status, kErrMbarTimeout, 602, 0);
  if (tr) tr[6] = globaltimer_ns();
  tc_fence_after();
  {
    const int t = tid & 127;
    const bool in = t < n && ok2;
    float* ut = a.uT + oidx * D * C;
    __nv_bfloat16* wd = a.w + (oidx * C + t) * D;
#pragma unroll 1
    for (int e = half * 64; e < half * 64 + 64; e += 16) {
      float u[16], w[16];
      if (ok2) {
        tmem_ld16(trow + e, u);
        tmem_ld16(trow + 128 + e, w);
        tmem_ld_wait();
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        u[i] = in ? u[i] : 0.f;
        w[i] = in ? w[i] : 0.f;
        ut[(int64_t)(e + i) * C + t] = u[i];  // U^T[d][t]: coalesced over t
      }
      *reinterpret_cast<uint4*>(wd + e) = pack8_bf16(w);
      *reinterpret_cast<uint4*>(wd + e + 8) = pack8_bf16(w + 8);
    }
    if (tid == 0) a.gC[oidx] = __expf(gcl);
  }
  if (tr) tr[7] = globaltimer_ns();
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tb, 256);
  }
}

// ------------------------------------------------------------------------------------------------
// Phase 2: grid (sequences, Hv), 160 threads: warps 0-3 epilogue (thread n = state column n, TMEM lane
// n), warp 4 lane 0 issues the MMAs. Epilogue thread 0 issues the TMA loads of the operand tiles.
// ------------------------------------------------------------------------------------------------
template <typename ST>
__global__ void __launch_bounds__(160, 1) gdn_chunk_scan_kernel(const __grid_constant__ CUtensorMap tmW,
                                                                const __grid_constant__ CUtensorMap tmQ,
                                                                const __grid_constant__ CUtensorMap tmK,
                                                                const __grid_constant__ CUtensorMap tmP,
                                                                ST* __restrict__ state, const ChunkArgs a) {
  using namespace gch;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* St = smem + P2_S;
  uint8_t* Dt = smem + P2_D;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + P2_BAR);  // W, gamma q landed
  uint64_t* full_b = full_a + 1;                                   // K-hat^T, P landed
  uint64_t* mma1 = full_a + 2;                                     // MMA1 + MMA2 done
  uint64_t* mma2 = full_a + 3;                                     // MMA3 + MMA4 done
  uint64_t* s_ready = full_a + 4;                                  // S^T operand written (128 arrivals)
  uint64_t* d_ready = full_a + 5;                                  // Delta^T operand written, S scaled
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + P2_BAR + 64);
  __shared__ volatile int s_abort;
  const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c0 = a.seq_chunk0[s], c1 = a.seq_chunk0[s + 1];
  const int slot = a.seq_slot[s];
  if (tid == 0) {
    mbar_init(full_a, 1);
    mbar_init(full_b, 1);
    mbar_init(mma1, 1);
    mbar_init(mma2, 1);
    mbar_init(s_ready, 128);
    mbar_init(d_ready, 128);
    fence_mbar_init();
    s_abort = 0;
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmP);
  }
  if (warp == 4) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *tmem_holder;
  constexpr uint32_t DACC = 0, OACC = 128, SM = 256;
  pdl_wait();  // phase 1 wrote the operands
  auto load_a = [&](int c) {
    const int row = (c * a.Hv + h) * C;
    mbar_arrive_expect_tx(full_a, 2 * TILE);
    tma_load_2d(smem + P2_W, &tmW, full_a, 0, row);
    tma_load_2d(smem + P2_W + REG, &tmW, full_a, 64, row);
    tma_load_2d(smem + P2_Q, &tmQ, full_a, 0, row);
    tma_load_2d(smem + P2_Q + REG, &tmQ, full_a, 64, row);
  };
  auto load_b = [&](int c) {
    const int row = (c * a.Hv + h) * C;
    mbar_arrive_expect_tx(full_b, 2 * TILE);
    tma_load_2d(smem + P2_K, &tmK, full_b, 0, row);
    tma_load_2d(smem + P2_K + REG, &tmK, full_b, 64, row);
    tma_load_2d(smem + P2_P, &tmP, full_b, 0, row);
    tma_load_2d(smem + P2_P + REG, &tmP, full_b, 64, row);
  };
  if (warp == 4) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      for (int c = c0; c < c1; ++c) {
        const uint32_t ph = (uint32_t)((c - c0) & 1);
        if (!mbar_wait(full_a, ph, a.timeout_ns) || !mbar_wait(s_ready, ph, a.timeout_ns)) {
          report_error(a.status, kErrMbarTimeout, 610, c);
          s_abort = 1;
          break;
        }
        tc_fence_after();
        mma_tile(tb + DACC, smem_u32(St), smem_u32(smem + P2_W), 0);
        mma_tile(tb + OACC, smem_u32(St), smem_u32(smem + P2_Q), 0);
        tc_commit(mma1);
        if (!mbar_wait(d_ready, ph, a.timeout_ns) || !mbar_wait(full_b, ph, a.timeout_ns)) {
          report_error(a.status, kErrMbarTimeout, 611, c);
          s_abort = 1;
          break;
        }
        tc_fence_after();
        mma_tile_mn(tb + SM, smem_u32(Dt), smem_u32(smem + P2_K), 1);  // K-hat rows: MN-major B
        mma_tile(tb + OACC, smem_u32(Dt), smem_u32(smem + P2_P), 1);
        tc_commit(mma2);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue warps ------------------------------
    const int nrow = tid;  // state column n = TMEM lane n
    const uint32_t trow = tb + ((uint32_t)((warp & 3) * 32) << 16);  // warps w and w + 4 share a lane quadrant
    ST* Sp = state + (((int64_t)slot * a.Hv + h) * D + nrow) * D;  // S^T row n (= state column n)
    const bool hs = a.seq_has_state[s] != 0;
    if (tid == 0 && c1 > c0) {
      load_a(c0);
      load_b(c0);
    }
    // initial state: TMEM master (fp32) and the bf16 operand
#pragma unroll 1
    for (int e = 0; e < D; e += 16) {
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = hs ? to_float(Sp[e + i]) : 0.f;
      tmem_st16(trow + SM + e, x);
      st_tile16(St, nrow, e, x);
    }
    tmem_st_wait();
    fence_proxy_async();
    tc_fence_before();
    mbar_arrive(s_ready);
    bool ok = true;
    for (int c = c0; c < c1 && ok; ++c) {
      const uint32_t ph = (uint32_t)((c - c0) & 1);
      const int t0 = a.ctab[3 * c], n = a.ctab[3 * c + 1];
      const int64_t oidx = (int64_t)c * a.Hv + h;
      const float* ur = a.uT + (oidx * D + nrow) * C;  // U^T row n
      const float gC = a.gC[oidx];
      // the U^T row is requested before waiting on the tensor cores, so its latency hides behind MMA1/2
      float4 uv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) uv[i] = *reinterpret_cast<const float4*>(ur + 4 * i);
      // ---- E1: Delta^T = U^T - S^T W^T; S^T *= gamma_C
      ok = __all_sync(0xffffffffu, mbar_wait(mma1, ph, a.timeout_ns)) && !s_abort;
      if (!ok) break;
      tc_fence_after();
      if (tid == 0 && c + 1 < c1) load_a(c + 1);  // W / gamma q buffers are free again
#pragma unroll
      for (int e = 0; e < C; e += 16) {
        float x[16], sm[16];
        tmem_ld16(trow + DACC + e, x);
        tmem_ld16(trow + SM + e, sm);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 u4 = uv[(e + i) >> 2];
          x[i] = u4.x - x[i]; x[i + 1] = u4.y - x[i + 1]; x[i + 2] = u4.z - x[i + 2]; x[i + 3] = u4.w - x[i + 3];
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) sm[i] *= gC;
        st_tile16(Dt, nrow, e, x);
        tmem_st16(trow + SM + e, sm);
      }
      tmem_st_wait();
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(d_ready);
      // ---- E2: O^T -> o; S^T -> next operand
      ok = __all_sync(0xffffffffu, mbar_wait(mma2, ph, a.timeout_ns)) && !s_abort;
      if (!ok) break;
      tc_fence_after();
      if (tid == 0 && c + 1 < c1) load_b(c + 1);
#pragma unroll 1
      for (int e = 0; e < C; e += 16) {
        float x[16];
        tmem_ld16(trow + OACC + e, x);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (e + i < n) a.o[((int64_t)(t0 + e + i) * a.Hv + h) * D + nrow] = x[i];
      }
      if (c + 1 < c1) {
#pragma unroll 1
        for (int e = 0; e < D; e += 16) {
          float x[16];
          tmem_ld16(trow + SM + e, x);
          tmem_ld_wait();
          st_tile16(St, nrow, e, x);
        }
        fence_proxy_async();
        tc_fence_before();
        mbar_arrive(s_ready);
      }
    }
    if (!ok) report_error(a.status, kErrMbarTimeout, 612, 0);
    if (ok && a.write_state) {
#pragma unroll 1
      for (int e = 0; e < D; e += 16) {
        float x[16];
        tmem_ld16(trow + SM + e, x);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) Sp[e + i] = from_float<ST>(x[i]);
      }
    }
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tb, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// host
// ------------------------------------------------------------------------------------------------
// qkv: bf16 [T, 2 Hk + Hv, 128] (q | k | v heads from gdn_conv_prep); g / beta fp32 [T, Hv]; ctab [chunks, 3]
// int32 (first token, tokens, sequence); seq_chunk0 [S + 1] int32; scratch: w, qg, kh, p bf16
// [chunks * Hv * 128, 128], uT fp32 [chunks * Hv * 128, 128], gC fp32 [chunks * Hv]; o fp32 [T, Hv, 128].
static unsigned long long* g_chunk_trace = nullptr;
static int64_t g_chunk_trace_cap = 0;
// tuning: 8 timestamps per phase-1 CTA of the next gdn_chunked calls into `buf` (None: off)
void gdn_chunk_trace(c10::optional<torch::Tensor> buf) {
  if (buf.has_value() && buf->defined()) {
    TORCH_CHECK(buf->is_cuda() && buf->dtype() == torch::kInt64 && buf->is_contiguous(), "gdn_chunk_trace: int64 cuda");
    g_chunk_trace = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
    g_chunk_trace_cap = buf->numel();
  } else {
    g_chunk_trace = nullptr;
    g_chunk_trace_cap = 0;
  }
}

void gdn_chunked(torch::Tensor qkv, torch::Tensor g, torch::Tensor beta, torch::Tensor state, torch::Tensor ctab,
                 torch::Tensor seq_chunk0, torch::Tensor seq_slot, torch::Tensor seq_has_state, bool write_state,
                 int64_t Hk, int64_t Hv, torch::Tensor w, torch::Tensor qg, torch::Tensor kh, torch::Tensor p,
                 torch::Tensor uT, torch::Tensor gC, torch::Tensor o, torch::Tensor status) {
  using namespace gch;
  const int64_t nchunks = ctab.size(0), S = seq_slot.size(0);
  if (nchunks == 0 || S == 0) return;
  const int64_t T = g.size(0), NH = 2 * Hk + Hv;
  TORCH_CHECK(qkv.dtype() == torch::kBFloat16 && qkv.is_contiguous() && qkv.numel() >= T * NH * D &&
                  (reinterpret_cast<uintptr_t>(qkv.data_ptr()) & 15) == 0,
              "gdn_chunked: qkv bf16 [T, 2 Hk + Hv, 128]");
  TORCH_CHECK(Hv % Hk == 0 && g.size(1) == Hv && o.size(1) == Hv && o.size(2) == D, "gdn_chunked: heads");
  TORCH_CHECK(state.size(1) == Hv && state.size(2) == D && state.size(3) == D, "gdn_chunked: state [slots, Hv, 128, 128]");
  TORCH_CHECK(ctab.dtype() == torch::kInt32 && ctab.size(1) == 3 && seq_chunk0.numel() == S + 1, "gdn_chunked: tables");
  const int64_t rows = nchunks * Hv * C;
  TORCH_CHECK(w.numel() >= rows * D && qg.numel() >= rows * D && kh.numel() >= rows * D && p.numel() >= rows * C &&
                  uT.numel() >= rows * C && gC.numel() >= nchunks * Hv,
              "gdn_chunked: scratch too small");
  for (auto* t : {&g, &beta, &o}) TORCH_CHECK(t->is_contiguous() && t->dtype() == torch::kFloat32, "gdn_chunked: fp32");
  const at::cuda::CUDAGuard guard(g.device());
  auto st = at::cuda::getCurrentCUDAStream();
  ChunkArgs a = {};
  a.g = g.data_ptr<float>(); a.beta = beta.data_ptr<float>();
  a.Hk = (int)Hk; a.Hv = (int)Hv;
  a.ctab = ctab.data_ptr<int32_t>(); a.nchunks = (int)nchunks;
  a.w = reinterpret_cast<__nv_bfloat16*>(w.data_ptr()); a.qg = reinterpret_cast<__nv_bfloat16*>(qg.data_ptr());
  a.kh = reinterpret_cast<__nv_bfloat16*>(kh.data_ptr()); a.p = reinterpret_cast<__nv_bfloat16*>(p.data_ptr());
  a.uT = uT.data_ptr<float>(); a.gC = gC.data_ptr<float>();
  a.seq_chunk0 = seq_chunk0.data_ptr<int32_t>(); a.seq_slot = seq_slot.data_ptr<int32_t>();
  a.seq_has_state = seq_has_state.data_ptr<int32_t>(); a.write_state = write_state ? 1 : 0;
  a.o = o.data_ptr<float>();
  a.status = status.data_ptr<int>();
  a.timeout_ns = 2000000000ull;
  a.trace = (nchunks * Hv * 8 <= g_chunk_trace_cap) ? g_chunk_trace : nullptr;
  // q|k|v copy as a 3-D map (128 elements, heads, tokens): a box is 64 elements x 1 head x 128 tokens
  CUtensorMap tqkv;
  {
    cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)NH, (cuuint64_t)T};
    cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)NH * D * 2};
    cuuint32_t box[3] = {64, 1, 128};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = get_encode_fn()(&tqkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, qkv.data_ptr(), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "gdn_chunked: q|k|v tensor map (", (int)r, ")");
  }
  TORCH_CHECK(ensure_smem_attr((const void*)gdn_chunk_prep_kernel, P1_SMEM) == cudaSuccess, "gdn_chunked: smem");
  TORCH_CHECK(launch_pdl(gdn_chunk_prep_kernel, dim3((unsigned)nchunks, (unsigned)Hv), dim3(256), (size_t)P1_SMEM, st,
                         tqkv, a) == cudaSuccess,
              "gdn_chunk_prep launch");
  const CUtensorMap tW = tmap_bf16_kmajor(w.data_ptr(), rows, D, D, 128);
  const CUtensorMap tQ = tmap_bf16_kmajor(qg.data_ptr(), rows, D, D, 128);
  const CUtensorMap tK = tmap_bf16_kmajor(kh.data_ptr(), rows, D, D, 128);
  const CUtensorMap tP = tmap_bf16_kmajor(p.data_ptr(), rows, C, C, 128);
#define R9K_GCS(ST_T)                                                                                             \
  {                                                                                                               \
    TORCH_CHECK(ensure_smem_attr((const void*)gdn_chunk_scan_kernel<ST_T>, P2_SMEM) == cudaSuccess, "gdn_chunked"); \
    TORCH_CHECK(launch_pdl(gdn_chunk_scan_kernel<ST_T>, dim3((unsigned)S, (unsigned)Hv), dim3(160), (size_t)P2_SMEM,  \
                           st, tW, tQ, tK, tP, reinterpret_cast<ST_T*>(state.data_ptr()), a) == cudaSuccess,         \
                "gdn_chunk_scan launch");                                                                         \
  }
  if (state.dtype() == torch::kFloat32) R9K_GCS(float) else R9K_GCS(__nv_bfloat16)
#undef R9K_GCS
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k
