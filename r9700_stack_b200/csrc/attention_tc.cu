// tcgen05 flash attention over the paged fp8 KV cache (sm_100a).
//
// One CTA = one KV head x one query tile of up to 128 rows, where a row is a (query token, q head of
// this KV head's GQA group) pair, so the G heads of a group share every K/V byte loaded. Two modes:
//   * decode / verify (mode 0): grid (seqs, kv heads, splits). A sequence's 1..21 query tokens form
//     the tile and the KV range [0, ctx) is cut into `nsplit` chunks of whole 128-key tiles; each split
//     writes an unnormalised partial (O, max, sum) that attn_combine merges.
//   * prefill (mode 1): grid (tiles, kv heads). A host table lists (sequence, first token, tokens) per
//     tile; each CTA covers the whole causal KV range and writes the final output directly.
// Reference counterparts: kernels/r9k_attn.hip:226-447 (paged causal prefill, fp8 KV) and the stock
// split-KV verify backend wrapped by r9700_vllm/attn/triton3d.py:125-290.
//
// Data path (all tiles 128-byte swizzled):
//   K, V pages -> TMA (2D map over [blocks * kv_heads * 64 rows, 256 B]) -> smem, e4m3 as stored.
//   Q rows -> e4m3 with a per-row scale, written into smem by the softmax warps.
//   S = Q K^T : tcgen05.mma kind::f8f6f4, M=128 (rows) N=128 (keys) K=256, accumulator in TMEM
//               (two S buffers so the next tile's QK^T overlaps this tile's softmax).
//   softmax  : one thread per row reads its S row from TMEM, P = exp2(s - m_ref) quantised to e4m3
//              into smem (m_ref lags the running max by up to 2^8, so P <= 256 fits e4m3; O is
//              rescaled in TMEM only when the max grows past that).
//   O += P V  : kind::f8f6f4 with V as an MN-major operand (d contiguous), N=256, O in TMEM.
// Warp roles: warp 0 TMA producer, warp 1 MMA issuer (TMEM owner), warps 2-5 softmax/epilogue.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "tmap.h"

namespace r9k {

namespace fa {
constexpr int D = 256;
constexpr int BLK = 64;          // KV page size (tokens)
constexpr int KT = 128;          // keys per tile (two pages)
constexpr int ROWS = 128;
constexpr int Q_BYTES = ROWS * D;            // e4m3, two 16 KB swizzle atoms (d halves)
constexpr int KV_TILE_BYTES = KT * D;        // 32 KB (two d-half atoms of 16 KB)
constexpr int P_BYTES = ROWS * KT;           // 16 KB
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_BYTES;       // 2 stages
constexpr int OFF_V = OFF_K + 2 * KV_TILE_BYTES;
constexpr int OFF_P = OFF_V + 2 * KV_TILE_BYTES;
constexpr int OFF_BAR = OFF_P + P_BYTES;
// barriers: q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], s_free[2], p_full, pv_done
constexpr int NBAR = 1 + 2 * 6 + 2;
constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
constexpr int SMEM = OFF_TMEM + 16 + 1024;
constexpr int TMEM_COLS = 512;   // O: [0,256), S0: [256,384), S1: [384,512)
constexpr int O_COL = 0, S_COL = 256;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: P <= 2^8
}  // namespace fa

struct AttnArgs {
  const __nv_bfloat16* q;  // [T, Hq, D]
  int Hq, Hkv, G;
  const int32_t* block_table;
  int max_blocks;
  const int32_t* tok_ctx;   // [T] visible keys of each query token (position + 1)
  const int32_t* seq_start; // mode 0: [S]
  const int32_t* seq_len;   // mode 0: [S]
  const int32_t* tile_tab;  // mode 1: [ntiles][3] = seq row, first token, tokens
  int ntiles;
  int mode;
  float scale_log2;         // sm_scale * k_scale * log2(e)
  float v_scale;
  // mode 0 outputs
  float* part_o;            // [T * Hq][nsplit][D]
  float* part_ml;           // [T * Hq][nsplit][2]
  int nsplit;
  // mode 1 outputs
  const __nv_bfloat16* gate;
  int64_t ld_gate;
  uint8_t* out_q;
  uint8_t* out_sf;
  int out_kblocks;
  __nv_bfloat16* out_bf16;
  int* status;
  uint64_t timeout_ns;
};

R9K_DEVINL uint64_t sdesc_mn_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// store 16 bytes into a 128-byte-swizzled K-major tile: row r, 16-byte chunk c
R9K_DEVINL void st_swz16(uint8_t* tile, int r, int c, uint4 v) {
  *reinterpret_cast<uint4*>(tile + r * 128 + ((c ^ (r & 7)) << 4)) = v;
}

R9K_DEVINL uint32_t pack4_e4m3(float a, float b, float c, float d) {
  const uint32_t lo = (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

__global__ void __launch_bounds__(192, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  pdl_wait();
  pdl_trigger();  // dependents may launch and prefetch while this grid runs
  using namespace fa;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 3;
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 7;
  uint64_t* s_full = bars + 9;
  uint64_t* s_free = bars + 11;
  uint64_t* p_full = bars + 13;
  uint64_t* pv_done = bars + 14;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);

  const int warp = warp_id(), lane = lane_id();
  const int kvh = blockIdx.y;

  // ---- work item ----
  int seq, tok0, ntok, kv0, kv1;
  if (a.mode == 0) {
    seq = blockIdx.x;
    tok0 = a.seq_start[seq];
    ntok = a.seq_len[seq];
    const int ctx = a.tok_ctx[tok0 + ntok - 1];
    // each sequence's key range is cut into nsplit chunks of a multiple of 128 keys
    const int chunk = ((ctx + a.nsplit - 1) / a.nsplit + KT - 1) / KT * KT;
    kv0 = blockIdx.z * chunk;
    kv1 = min(ctx, kv0 + chunk);
  } else {
    if ((int)blockIdx.x >= a.ntiles) return;
    seq = a.tile_tab[blockIdx.x * 3 + 0];
    tok0 = a.tile_tab[blockIdx.x * 3 + 1];
    ntok = a.tile_tab[blockIdx.x * 3 + 2];
    kv0 = 0;
    kv1 = a.tok_ctx[tok0 + ntok - 1];
  }
  const int nrows = min(ROWS, ntok * a.G);
  const int ntiles = kv1 > kv0 ? (kv1 - kv0 + KT - 1) / KT : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    fence_mbar_init();
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const int32_t* bt = a.block_table + (int64_t)seq * a.max_blocks;

  if (warp == 0) {
    // ------------------------------------ producer ------------------------------------
    if (lane == 0) {
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1;
        const uint32_t ph = (uint32_t)((j >> 1) & 1);
        const int key0 = kv0 + j * KT;
        int blk[2];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int pi = key0 / BLK + p;
          blk[p] = (pi < a.max_blocks && key0 + p * BLK < kv1) ? bt[pi] : 0;
        }
        if (!mbar_wait(&k_empty[s], ph ^ 1u, a.timeout_ns)) { report_error(a.status, kErrMbarTimeout, 200, j); break; }
        uint8_t* ks = smem + OFF_K + s * KV_TILE_BYTES;
        mbar_arrive_expect_tx(&k_full[s], KV_TILE_BYTES);
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_2d(ks + h * (KT * 128) + p * (BLK * 128), &tmK, &k_full[s], h * 128, (blk[p] * a.Hkv + kvh) * BLK);
        if (!mbar_wait(&v_empty[s], ph ^ 1u, a.timeout_ns)) { report_error(a.status, kErrMbarTimeout, 201, j); break; }
        uint8_t* vs = smem + OFF_V + s * KV_TILE_BYTES;
        mbar_arrive_expect_tx(&v_full[s], KV_TILE_BYTES);
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_2d(vs + h * (KT * 128) + p * (BLK * 128), &tmV, &v_full[s], h * 128, (blk[p] * a.Hkv + kvh) * BLK);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------ MMA issuer ------------------------------------
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t idesc_s = idesc_dense(kFmtE4M3, kFmtE4M3, ROWS, KT);
      constexpr uint32_t idesc_o = idesc_dense(kFmtE4M3, kFmtE4M3, ROWS, D) | (1u << 16);  // B (V) MN-major
      const uint32_t sq = smem_u32(smem + OFF_Q);
      const uint32_t sp = smem_u32(smem + OFF_P);
      bool ok = mbar_wait(q_full, 0, a.timeout_ns);
      if (!ok) report_error(a.status, kErrMbarTimeout, 210, 0);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        const uint32_t ph = (uint32_t)((j >> 1) & 1);
        if (!mbar_wait(&k_full[s], ph, a.timeout_ns)) return false;
        if (!mbar_wait(&s_free[s], ph ^ 1u, a.timeout_ns)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + OFF_K + s * KV_TILE_BYTES);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f8f6f4_ss(tbase + S_COL + s * KT, sdesc_k_sw128(sq + h * (ROWS * 128) + 32 * k),
                          sdesc_k_sw128(sk + h * (KT * 128) + 32 * k), idesc_s, (h > 0 || k > 0) ? 1u : 0u);
        tc_commit(&s_full[s]);
        tc_commit(&k_empty[s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles && !issue_s(j + 1)) { ok = false; break; }
        const int s = j & 1;
        if (!mbar_wait(p_full, (uint32_t)(j & 1), a.timeout_ns)) { ok = false; break; }
        if (!mbar_wait(&v_full[s], (uint32_t)((j >> 1) & 1), a.timeout_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + OFF_V + s * KV_TILE_BYTES);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f8f6f4_ss(tbase + O_COL, sdesc_k_sw128(sp + 32 * k), sdesc_mn_sw128(sv + k * 4096, KT * 128, 1024),
                        idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        tc_commit(pv_done);
        tc_commit(&v_empty[s]);
      }
      if (!ok) report_error(a.status, kErrMbarTimeout, 211, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------ softmax / epilogue ------------------------------------
    const int q = warp & 3;
    const int r = q * 32 + lane;  // TMEM lane == tile row
    const bool valid = r < nrows;
    const int rt = r / a.G, rg = r % a.G;
    const int tok = tok0 + rt;
    const int head = kvh * a.G + rg;
    const int ctx = valid ? a.tok_ctx[tok] : 0;
    // Q row -> e4m3 with per-row scale, into the swizzled Q tile
    float qscale = 1.f;
    {
      uint8_t* sq = smem + OFF_Q;
      float amax = 0.f;
      const __nv_bfloat16* qr = a.q + ((int64_t)tok * a.Hq + head) * D;
      if (valid) {
        for (int c = 0; c < D / 8; ++c) {
          const uint4 raw = reinterpret_cast<const uint4*>(qr)[c];
          const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
          for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(__bfloat162float(e[i])));
        }
      }
      qscale = amax > 0.f ? amax / 448.f : 1.f;
      const float inv = 1.f / qscale;
      for (int c = 0; c < D / 16; ++c) {  // 16 elements -> 16 bytes
        uint4 w = make_uint4(0, 0, 0, 0);
        if (valid) {
          const uint4 r0 = reinterpret_cast<const uint4*>(qr)[2 * c];
          const uint4 r1 = reinterpret_cast<const uint4*>(qr)[2 * c + 1];
          const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&r0);
          const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&r1);
          float f[16];
#pragma unroll
          for (int i = 0; i < 8; ++i) { f[i] = __bfloat162float(e0[i]) * inv; f[8 + i] = __bfloat162float(e1[i]) * inv; }
          w.x = pack4_e4m3(f[0], f[1], f[2], f[3]);
          w.y = pack4_e4m3(f[4], f[5], f[6], f[7]);
          w.z = pack4_e4m3(f[8], f[9], f[10], f[11]);
          w.w = pack4_e4m3(f[12], f[13], f[14], f[15]);
        }
        const int h = c / 8, cc = c % 8;
        st_swz16(sq + h * (ROWS * 128), r, cc, w);
      }
      fence_proxy_async();
      mbar_arrive(q_full);
    }
    const float sl2 = a.scale_log2 * qscale;
    float m_ref = -INFINITY, l = 0.f;
    const uint32_t trow = tbase + ((uint32_t)(q * 32) << 16);
    uint8_t* sp = smem + OFF_P;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[s], (uint32_t)((j >> 1) & 1), a.timeout_ns));
      if (!ok) break;
      tc_fence_after();
      float sv[KT];
#pragma unroll
      for (int c = 0; c < KT; c += 16) tmem_ld16(trow + S_COL + s * KT + c, sv + c);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_free[s]);
      const int key0 = kv0 + j * KT;
      float tmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < KT; ++c) {
        const int key = key0 + c;
        const bool vis = valid && key < ctx && key < kv1;
        sv[c] = vis ? sv[c] * sl2 : -INFINITY;
        tmax = fmaxf(tmax, sv[c]);
      }
      // the P buffer and O must be free: PV of the previous tile has completed
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (uint32_t)((j - 1) & 1), a.timeout_ns));
        if (!ok) break;
        tc_fence_after();
      }
      // O is rescaled only when some row's max grew past the threshold; the decision is made per
      // warp because tcgen05.ld/st are warp-collective
      const bool need = (m_ref != -INFINITY) && (tmax > m_ref + RESCALE_THRESHOLD);
      if (__any_sync(0xffffffffu, need)) {
        const float f = need ? exp2f(m_ref - tmax) : 1.f;
#pragma unroll 1
        for (int c = 0; c < D; c += 16) {
          float o[16];
          tmem_ld16(trow + O_COL + c, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] *= f;
          tmem_st16(trow + O_COL + c, o);
        }
        tmem_st_wait();
        if (need) l *= f;
      }
      if (need || (m_ref == -INFINITY && tmax != -INFINITY)) m_ref = tmax;
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < KT; c += 16) {
        float p[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          p[i] = (sv[c + i] == -INFINITY) ? 0.f : exp2f(sv[c + i] - m_ref);
          lsum += p[i];
        }
        uint4 w;
        w.x = pack4_e4m3(p[0], p[1], p[2], p[3]);
        w.y = pack4_e4m3(p[4], p[5], p[6], p[7]);
        w.z = pack4_e4m3(p[8], p[9], p[10], p[11]);
        w.w = pack4_e4m3(p[12], p[13], p[14], p[15]);
        st_swz16(sp, r, c / 16, w);
      }
      l += lsum;
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // ---- epilogue ----
    if (ok && ntiles > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (uint32_t)((ntiles - 1) & 1), a.timeout_ns));
      tc_fence_after();
    }
    if (!ok) report_error(a.status, kErrMbarTimeout, 220, r);
    if (a.mode == 0) {
      const int64_t pidx = ((int64_t)tok * a.Hq + head) * a.nsplit + blockIdx.z;
      const bool have = ntiles > 0 && ok;  // warp-uniform
      if (have) {
        float* po = a.part_o + pidx * D;
#pragma unroll 1
        for (int c = 0; c < D; c += 16) {
          float o[16];
          tmem_ld16(trow + O_COL + c, o);
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<float4*>(po + c + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
          }
        }
      }
      if (valid) {
        a.part_ml[pidx * 2 + 0] = have ? m_ref : -INFINITY;
        a.part_ml[pidx * 2 + 1] = have ? l : 0.f;
      }
    } else {
      const float inv_l = (l > 0.f) ? a.v_scale / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < D && ok && ntiles > 0; c += 32) {
        float o[32];
        tmem_ld16(trow + O_COL + c, o);
        tmem_ld16(trow + O_COL + c + 16, o + 16);
        tmem_ld_wait();
        if (!valid) continue;
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float v = o[i] * inv_l;
          if (a.gate != nullptr) v *= sigmoid_f(__bfloat162float(a.gate[(int64_t)tok * a.ld_gate + head * D + c + i]));
          v = __bfloat162float(__float2bfloat16(v));
          o[i] = v;
          am = fmaxf(am, fabsf(v));
        }
        const int64_t obase = (int64_t)tok * a.Hq * D + head * D + c;
        if (a.out_bf16 != nullptr) {
#pragma unroll
          for (int i = 0; i < 32; ++i) a.out_bf16[obase + i] = __float2bfloat16(o[i]);
        }
        if (a.out_q != nullptr) {
          const int e = mx_exponent(am, 448.f);
          const float si = exp2i(-e);
          uint32_t* dst = reinterpret_cast<uint32_t*>(a.out_q + obase);
#pragma unroll
          for (int i = 0; i < 32; i += 4) dst[i / 4] = pack4_e4m3(o[i] * si, o[i + 1] * si, o[i + 2] * si, o[i + 3] * si);
          a.out_sf[sf_offset(tok, (head * D + c) >> 5, a.out_kblocks)] = (uint8_t)(e + 127);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, fa::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------
// Decode / verify attention with keys on the MMA's M side ("swap-AB"): S^T = K Q^T and O^T += V^T P^T.
//
// A decode query tile is only ntok x G rows (6 for GQA 24/4), so the row-tile kernel above spends a
// 128-row MMA and 128 softmax threads per 6 useful rows. Here the 128 keys of a tile are the M = 128
// rows and the query rows are the N = 16..48 columns: S^T [keys x rows] lands in TMEM with one key per
// TMEM lane, each softmax thread owns one key and walks only the valid columns, and the per-column
// max / sum reduce across the 128 threads. P^T [rows x keys] (e4m3) is the B operand of O^T += V^T P^T,
// where V^T is V read as an MN-major A operand (d contiguous), two 128-row halves of d. Three K/V stages
// (192 KB) stay in flight per SM; S and P are double-buffered so QK^T and PV overlap the softmax.
// Columns keep their own running max with the same lazy rescale (threshold 2^8) as the row-tile
// kernel; partials go to attn_combine_kernel unchanged.
// ------------------------------------------------------------------------------------------------
namespace fd {
constexpr int D = 256, BLK = 64, KT = 128, NMAX = 48, STAGES = 3;
constexpr int Q_BYTES = 2 * NMAX * 128;   // two d-half atom columns of NMAX rows
constexpr int KV_TILE = KT * D;           // 32 KB
constexpr int P_BYTES = NMAX * 128;       // one atom column of NMAX rows (keys along K)
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_BYTES;
constexpr int OFF_V = OFF_K + STAGES * KV_TILE;
constexpr int OFF_P = OFF_V + STAGES * KV_TILE;
constexpr int OFF_RED = OFF_P + 2 * P_BYTES;        // float [2 parities][max, sum][4 warps][NMAX]
constexpr int OFF_COL = OFF_RED + 2 * 2 * 4 * NMAX * 4; // float sl2[NMAX], int ctx[NMAX]
constexpr int OFF_BAR = OFF_COL + 2 * NMAX * 4;
// q_full, k_full[3], k_empty[3], v_full[3], v_empty[3], s_full[2], s_free[2], p_full[2], pv_done[2]
constexpr int NBAR = 1 + 4 * STAGES + 8;
constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
constexpr int SMEM = OFF_TMEM + 16 + 1024;
constexpr int TMEM_COLS = 256;  // S buffers [0, 96), O^T halves [128, 224)
constexpr int S_COL = 0, O_COL = 128;
constexpr float RESCALE_THRESHOLD = 8.0f;
static_assert(SMEM <= 232448, "decode attention: shared memory");
}  // namespace fd

R9K_DEVINL void softmax_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// NC: compile-time bound on the query rows (columns) a tile carries, so the per-column loops of the
// softmax stay short and fully unrolled (8 for plain decode up to GQA 8, 48 for speculative verify)
template <int NC>
__global__ void __launch_bounds__(192, 1)
    attn_dec_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  using namespace fd;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + STAGES;
  uint64_t* v_full = k_empty + STAGES;
  uint64_t* v_empty = v_full + STAGES;
  uint64_t* s_full = v_empty + STAGES;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);
  float* red_base = reinterpret_cast<float*>(smem + OFF_RED);  // [parity][max | sum][4 warps][NMAX]
  float* col_sl2 = reinterpret_cast<float*>(smem + OFF_COL);
  int* col_ctx = reinterpret_cast<int*>(col_sl2 + NMAX);
  __shared__ int s_fail;  // a softmax warp's wait ran out: all four leave the loop together

  const int warp = warp_id(), lane = lane_id();
  const int kvh = blockIdx.y;
  const int seq = blockIdx.x;
  const int tok0 = a.seq_start[seq], ntok = a.seq_len[seq];
  const int ctx_last = a.tok_ctx[tok0 + ntok - 1];
  const int chunk = ((ctx_last + a.nsplit - 1) / a.nsplit + KT - 1) / KT * KT;
  const int kv0 = blockIdx.z * chunk, kv1 = min(ctx_last, kv0 + chunk);
  const int NQ = min(NC, ntok * a.G);
  const int N = (NQ + 15) / 16 * 16;
  const int ntiles = kv1 > kv0 ? (kv1 - kv0 + KT - 1) / KT : 0;

  if (threadIdx.x == 0) {
    s_fail = 0;
    mbar_init(q_full, 128);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128);
      mbar_init(&p_full[s], 128);
      mbar_init(&pv_done[s], 1);
    }
    fence_mbar_init();
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const int32_t* bt = a.block_table + (int64_t)seq * a.max_blocks;

  if (warp == 0) {
    // ------------------------------------ producer ------------------------------------
    if (lane == 0) {
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % STAGES;
        const uint32_t ph = (uint32_t)((j / STAGES) & 1);
        const int key0 = kv0 + j * KT;
        int blk[2];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int pi = key0 / BLK + p;
          blk[p] = (pi < a.max_blocks && key0 + p * BLK < kv1) ? bt[pi] : 0;
        }
        if (!mbar_wait(&k_empty[st], ph ^ 1u, a.timeout_ns)) { report_error(a.status, kErrMbarTimeout, 230, j); break; }
        uint8_t* ks = smem + OFF_K + st * KV_TILE;
        mbar_arrive_expect_tx(&k_full[st], KV_TILE);
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_2d(ks + h * (KT * 128) + p * (BLK * 128), &tmK, &k_full[st], h * 128, (blk[p] * a.Hkv + kvh) * BLK);
        if (!mbar_wait(&v_empty[st], ph ^ 1u, a.timeout_ns)) { report_error(a.status, kErrMbarTimeout, 231, j); break; }
        uint8_t* vs = smem + OFF_V + st * KV_TILE;
        mbar_arrive_expect_tx(&v_full[st], KV_TILE);
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_2d(vs + h * (KT * 128) + p * (BLK * 128), &tmV, &v_full[st], h * 128, (blk[p] * a.Hkv + kvh) * BLK);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------ MMA issuer ------------------------------------
    if (lane == 0 && ntiles > 0) {
      const uint32_t idesc_s = idesc_dense(kFmtE4M3, kFmtE4M3, KT, N);
      const uint32_t idesc_o = idesc_dense(kFmtE4M3, kFmtE4M3, 128, N) | (1u << 15);  // A (V^T) MN-major
      const uint32_t sq = smem_u32(smem + OFF_Q);
      bool ok = mbar_wait(q_full, 0, a.timeout_ns);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1, st = j % STAGES;
        if (!mbar_wait(&k_full[st], (uint32_t)((j / STAGES) & 1), a.timeout_ns)) return false;
        if (!mbar_wait(&s_free[s], (uint32_t)(((j >> 1) & 1) ^ 1), a.timeout_ns)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + OFF_K + st * KV_TILE);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f8f6f4_ss(tbase + S_COL + s * NMAX, sdesc_k_sw128(sk + h * (KT * 128) + 32 * k),
                          sdesc_k_sw128(sq + h * (NMAX * 128) + 32 * k), idesc_s, (h > 0 || k > 0) ? 1u : 0u);
        tc_commit(&s_full[s]);
        tc_commit(&k_empty[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles && !issue_s(j + 1)) { ok = false; break; }
        const int pb = j & 1, st = j % STAGES;
        if (!mbar_wait(&p_full[pb], (uint32_t)((j >> 1) & 1), a.timeout_ns)) { ok = false; break; }
        if (!mbar_wait(&v_full[st], (uint32_t)((j / STAGES) & 1), a.timeout_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + OFF_V + st * KV_TILE);
        const uint32_t sp = smem_u32(smem + OFF_P + pb * P_BYTES);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f8f6f4_ss(tbase + O_COL + h * NMAX, sdesc_mn_sw128(sv + h * (KT * 128) + k * 4096, KT * 128, 1024),
                          sdesc_k_sw128(sp + 32 * k), idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        tc_commit(&pv_done[pb]);
        tc_commit(&v_empty[st]);
      }
      if (!ok) report_error(a.status, kErrMbarTimeout, 232, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------ softmax / epilogue ------------------------------------
    const int q = warp & 3;
    const int r = q * 32 + lane;  // TMEM lane == key within the tile
    const int tr = threadIdx.x - 64;  // 0..127 for the per-row set-up
    // zero both P buffers (rows >= NQ stay zero), then the Q rows and per-column constants
    for (int i = tr; i < 2 * P_BYTES / 16; i += 128) reinterpret_cast<uint4*>(smem + OFF_P)[i] = make_uint4(0, 0, 0, 0);
    {
      uint8_t* sq = smem + OFF_Q;
      const int n = tr;
      if (n < N) {
        const bool valid = n < NQ;
        const int tok = tok0 + n / a.G, head = kvh * a.G + n % a.G;
        const __nv_bfloat16* qr = a.q + ((int64_t)tok * a.Hq + head) * D;
        float amax = 0.f;
        if (valid)
          for (int c = 0; c < D / 8; ++c) {
            const uint4 raw = reinterpret_cast<const uint4*>(qr)[c];
            const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(__bfloat162float(e[i])));
          }
        const float qscale = amax > 0.f ? amax / 448.f : 1.f, inv = 1.f / qscale;
        for (int c = 0; c < D / 16; ++c) {
          uint4 w = make_uint4(0, 0, 0, 0);
          if (valid) {
            const uint4 r0 = reinterpret_cast<const uint4*>(qr)[2 * c];
            const uint4 r1 = reinterpret_cast<const uint4*>(qr)[2 * c + 1];
            const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&r0);
            const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&r1);
            float f[16];
#pragma unroll
            for (int i = 0; i < 8; ++i) { f[i] = __bfloat162float(e0[i]) * inv; f[8 + i] = __bfloat162float(e1[i]) * inv; }
            w.x = pack4_e4m3(f[0], f[1], f[2], f[3]);
            w.y = pack4_e4m3(f[4], f[5], f[6], f[7]);
            w.z = pack4_e4m3(f[8], f[9], f[10], f[11]);
            w.w = pack4_e4m3(f[12], f[13], f[14], f[15]);
          }
          st_swz16(sq + (c / 8) * (NMAX * 128), n, c % 8, w);
        }
        col_sl2[n] = a.scale_log2 * qscale;
        col_ctx[n] = valid ? a.tok_ctx[tok] : 0;
      }
      fence_proxy_async();
      mbar_arrive(q_full);
    }
    softmax_bar();
    constexpr int NCP = (NC + 15) / 16 * 16;  // register columns, whole 16-column TMEM loads
    // columns past NQ carry context 0: every key is masked, so they need no branches
    float mref[NC], lsum_tot[NC], csl2[NC];
    int cctx[NC];
#pragma unroll
    for (int n = 0; n < NC; ++n) {
      mref[n] = -INFINITY;
      lsum_tot[n] = 0.f;
      csl2[n] = n < N ? col_sl2[n] : 0.f;
      cctx[n] = n < N ? col_ctx[n] : 0;
    }
    bool ok = true;
    // every softmax thread runs the same barriers each tile; a wait that runs out only raises s_fail,
    // and the loop is left at the end of the tile, where all four warps see it together
    for (int j = 0; j < ntiles; ++j) {
      const int s = j & 1, pb = j & 1;
      bool w_ok = __all_sync(0xffffffffu, mbar_wait(&s_full[s], (uint32_t)((j >> 1) & 1), a.timeout_ns));
      tc_fence_after();
      float sv[NCP];
      const uint32_t trow = tbase + ((uint32_t)(q * 32) << 16) + S_COL + s * NMAX;
#pragma unroll
      for (int c = 0; c < NCP; c += 16)
        if (c < N) tmem_ld16(trow + c, sv + c);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_free[s]);
      const int key = kv0 + j * KT + r;
      float* red_max = red_base + (j & 1) * 8 * NMAX;
      float* red_sum = red_max + 4 * NMAX;
      // masked, scaled scores and per-warp column maxima (the NC columns reduce side by side)
      float mx[NC];
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        const bool vis = key < cctx[n] && key < kv1;
        sv[n] = vis ? sv[n] * csl2[n] : -INFINITY;
        mx[n] = sv[n];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int n = 0; n < NC; ++n) mx[n] = fmaxf(mx[n], __shfl_xor_sync(0xffffffffu, mx[n], o));
      if (lane == 0) {  // the butterfly left every lane with all NC column maxima
#pragma unroll
        for (int n = 0; n < NC; ++n) red_max[q * NMAX + n] = mx[n];
      }
      softmax_bar();
      // new references (identical in every thread) and the columns whose O must be rescaled
      float fac[NCP];
      bool any = false;
#pragma unroll
      for (int n = 0; n < NCP; ++n) fac[n] = 1.f;
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        fac[n] = 1.f;
        if (n < NQ) {
          const float tmax = fmaxf(fmaxf(red_max[n], red_max[NMAX + n]), fmaxf(red_max[2 * NMAX + n], red_max[3 * NMAX + n]));
          const bool need = mref[n] != -INFINITY && tmax > mref[n] + RESCALE_THRESHOLD;
          if (need) {
            fac[n] = exp2f(mref[n] - tmax);
            any = true;
          }
          if (need || (mref[n] == -INFINITY && tmax != -INFINITY)) mref[n] = tmax;
        }
      }
      // P buffer pb is free once the PV of tile j - 2 has completed; O must be complete before a rescale
      if (j >= 2)
        w_ok &= __all_sync(0xffffffffu, mbar_wait(&pv_done[pb], (uint32_t)(((j - 2) >> 1) & 1), a.timeout_ns));
      if (any && j >= 1) {
        w_ok &= __all_sync(0xffffffffu, mbar_wait(&pv_done[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1), a.timeout_ns));
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t orow = tbase + ((uint32_t)(q * 32) << 16) + O_COL + h * NMAX;
#pragma unroll
          for (int c = 0; c < NCP; c += 16) {
            if (c < N) {
              float o[16];
              tmem_ld16(orow + c, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] *= fac[c + i];
              tmem_st16(orow + c, o);
            }
          }
        }
        tmem_st_wait();
      }
      // P^T row n, key r (byte r of row n in the 128-byte swizzled atom column)
      uint8_t* prow = smem + OFF_P + pb * P_BYTES;
      float ps[NC];
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        const float p = sv[n] == -INFINITY ? 0.f : exp2f(sv[n] - mref[n]);
        const __nv_fp8_e4m3 e(p);
        prow[n * 128 + ((((r >> 4) ^ (n & 7)) << 4) | (r & 15))] = e.__x;
        ps[n] = p;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int n = 0; n < NC; ++n) ps[n] += __shfl_xor_sync(0xffffffffu, ps[n], o);
      if (lane == 0) {
#pragma unroll
        for (int n = 0; n < NC; ++n) red_sum[q * NMAX + n] = ps[n];
      }
      if (!w_ok && lane == 0) atomicOr(&s_fail, 1);
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&p_full[pb]);
      softmax_bar();
#pragma unroll
      for (int n = 0; n < NC; ++n)
        lsum_tot[n] = lsum_tot[n] * fac[n] + ((red_sum[n] + red_sum[NMAX + n]) + (red_sum[2 * NMAX + n] + red_sum[3 * NMAX + n]));
      if (s_fail) {
        ok = false;
        break;
      }
      // the reduction buffers alternate by tile parity: this tile's are rewritten two tiles later,
      // after both barriers of the next tile
    }
    // ---- epilogue: O^T row d = h * 128 + r of every valid column ----
    if (ok && ntiles > 0) {
      const int jl = ntiles - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[jl & 1], (uint32_t)((jl >> 1) & 1), a.timeout_ns));
      tc_fence_after();
    }
    if (!ok) report_error(a.status, kErrMbarTimeout, 233, r);
    const bool have = ntiles > 0 && ok;
    if (have) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t orow = tbase + ((uint32_t)(q * 32) << 16) + O_COL + h * NMAX;
#pragma unroll
        for (int c = 0; c < NCP; c += 16) {
          if (c < N) {
            float o[16];
            tmem_ld16(orow + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int n = c + i;
              if (n < NQ) {
                const int tok = tok0 + n / a.G, head = kvh * a.G + n % a.G;
                const int64_t pidx = ((int64_t)tok * a.Hq + head) * a.nsplit + blockIdx.z;
                a.part_o[pidx * D + h * 128 + r] = o[i];
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int n = 0; n < NC; ++n) {
      if (n < NQ && tr == n) {
        const int tok = tok0 + n / a.G, head = kvh * a.G + n % a.G;
        const int64_t pidx = ((int64_t)tok * a.Hq + head) * a.nsplit + blockIdx.z;
        a.part_ml[pidx * 2 + 0] = have ? mref[n] : -INFINITY;
        a.part_ml[pidx * 2 + 1] = have ? lsum_tot[n] : 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, fd::TMEM_COLS);
  }
}

// merge split-KV partials, apply the output gate, write bf16 and/or MXFP8. One warp per (token, head):
// lane s holds split s's (max, sum), so the global max and the weighted sum are two shuffle
// reductions, and the partial rows are requested four splits at a time (independent loads in flight
// instead of one dependent read per split). Empty splits (sum 0) get weight 0 and are selected away,
// so whatever their partial rows hold never reaches the output.
__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int T, int Hq,
                                    int nsplit, float v_scale, const __nv_bfloat16* __restrict__ gate, int64_t ld_gate,
                                    __nv_bfloat16* __restrict__ out_bf16, uint8_t* __restrict__ out_q,
                                    uint8_t* __restrict__ out_sf, int out_kblocks) {
  pdl_wait();
  pdl_trigger();  // the next GEMM may start streaming its weights
  constexpr int D = fa::D;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)T * Hq) return;
  const int tok = (int)(gw / Hq), head = (int)(gw % Hq);
  const float* ml = part_ml + gw * nsplit * 2;
  float m_l = -INFINITY, l_l = 0.f;
  if (lane < nsplit) {
    const float2 v = *reinterpret_cast<const float2*>(ml + 2 * lane);
    m_l = v.x;
    l_l = v.y;
  }
  const bool live = l_l > 0.f && m_l != -INFINITY;
  float M = live ? m_l : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float w_l = live ? exp2f(m_l - M) : 0.f;
  float L = w_l * l_l;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  const float* po0 = part_o + gw * nsplit * D + lane;
#pragma unroll 4
  for (int s = 0; s < nsplit; ++s) {
    const float w = __shfl_sync(0xffffffffu, w_l, s);
    const float* po = po0 + (int64_t)s * D;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float p = po[32 * i];
      acc[i] += w > 0.f ? w * p : 0.f;
    }
  }
  const float inv = L > 0.f ? v_scale / L : 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    float o = acc[i] * inv;
    if (gate != nullptr) o *= sigmoid_f(__bfloat162float(gate[(int64_t)tok * ld_gate + head * D + d]));
    o = __bfloat162float(__float2bfloat16(o));
    if (out_bf16 != nullptr) out_bf16[(int64_t)tok * Hq * D + head * D + d] = __float2bfloat16(o);
    if (out_q != nullptr) {
      float am = fabsf(o);
      for (int s2 = 16; s2 > 0; s2 >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, s2));
      const int e = mx_exponent(am, 448.f);
      out_q[(int64_t)tok * Hq * D + head * D + d] = f32_to_e4m3(o * exp2i(-e));
      if (lane == 0) out_sf[sf_offset(tok, (head * D + 32 * i) >> 5, out_kblocks)] = (uint8_t)(e + 127);
    }
  }
}

static void attn_tc_launch(const AttnArgs& a, const CUtensorMap& tk, const CUtensorMap& tv, dim3 grid, cudaStream_t st) {
  TORCH_CHECK(ensure_smem_attr((const void*)attn_tc_kernel, fa::SMEM) == cudaSuccess, "attn_tc: smem attribute");
  TORCH_CHECK(launch_pdl(attn_tc_kernel, grid, dim3(192), (size_t)fa::SMEM, st, tk, tv, a) == cudaSuccess, "attn_tc launch");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static AttnArgs base_args(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& block_table,
                          const torch::Tensor& tok_ctx, double sm_scale, double k_scale, double v_scale,
                          const torch::Tensor& status) {
  AttnArgs a = {};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.Hq = (int)q.size(1);
  a.Hkv = (int)kc.size(1);
  a.G = a.Hq / a.Hkv;
  TORCH_CHECK(a.Hq % a.Hkv == 0, "attn_tc: Hq % Hkv");
  TORCH_CHECK(q.size(2) == fa::D && kc.size(3) == fa::D && kc.size(2) == fa::BLK, "attn_tc: head_dim 256, page 64");
  a.block_table = block_table.data_ptr<int32_t>();
  a.max_blocks = (int)block_table.size(1);
  a.tok_ctx = tok_ctx.data_ptr<int32_t>();
  a.scale_log2 = (float)(sm_scale * k_scale * 1.4426950408889634);
  a.v_scale = (float)v_scale;
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
  return a;
}

static CUtensorMap kv_tmap(const torch::Tensor& c) {
  const int64_t rows = c.size(0) * c.size(1) * c.size(2);
  return tmap_u8_kmajor(c.data_ptr(), rows, fa::D, fa::BLK);
}

static bool dec_kernel_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("R9K_ATTN_DEC");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// decode / verify: split-KV partials + combine
void attn_tc_decode(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                    torch::Tensor tok_ctx, torch::Tensor seq_start, torch::Tensor seq_len, double sm_scale,
                    double k_scale, double v_scale, torch::Tensor part_o, torch::Tensor part_ml,
                    c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> out,
                    c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_sf, torch::Tensor status,
                    int64_t max_rows) {
  const int64_t T = q.size(0), S = seq_start.size(0);
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  AttnArgs a = base_args(q, k_cache, block_table, tok_ctx, sm_scale, k_scale, v_scale, status);
  a.mode = 0;
  a.seq_start = seq_start.data_ptr<int32_t>();
  a.seq_len = seq_len.data_ptr<int32_t>();
  a.nsplit = (int)part_ml.size(1);
  TORCH_CHECK(a.nsplit >= 1 && a.nsplit <= 32, "attn_tc: 1..32 KV splits (the combine keeps one split per lane)");
  TORCH_CHECK(part_o.size(0) >= T * a.Hq && part_o.size(1) == a.nsplit && part_o.size(2) == fa::D && part_o.is_contiguous() &&
                  part_ml.is_contiguous(), "attn_tc: part_o / part_ml must be contiguous [T*Hq, nsplit, ...]");
  TORCH_CHECK(seq_start.size(0) == S && S <= 65535, "attn_tc: seq count");
  a.part_o = part_o.data_ptr<float>();
  a.part_ml = part_ml.data_ptr<float>();
  auto st = at::cuda::getCurrentCUDAStream();
  // rows of the widest query tile: the caller's bound, else every token in one sequence
  const int64_t rows_bound = (max_rows > 0 ? max_rows : (T - S + 1)) * a.G;
  // up to 16 query rows per tile: keys-on-M kernel (its per-column registers grow with the rows);
  // wider verify tiles: the row-tile kernel
  if (rows_bound <= 16 && dec_kernel_enabled()) {
    auto kern = rows_bound <= 8 ? attn_dec_kernel<8> : attn_dec_kernel<16>;
    TORCH_CHECK(ensure_smem_attr((const void*)kern, fd::SMEM) == cudaSuccess, "attn_dec: smem attribute");
    TORCH_CHECK(launch_pdl(kern, dim3((unsigned)S, (unsigned)a.Hkv, (unsigned)a.nsplit), dim3(192), (size_t)fd::SMEM,
                           st, kv_tmap(k_cache), kv_tmap(v_cache), a) == cudaSuccess, "attn_dec launch");
  } else {
    attn_tc_launch(a, kv_tmap(k_cache), kv_tmap(v_cache), dim3((unsigned)S, (unsigned)a.Hkv, (unsigned)a.nsplit), st);
  }
  const __nv_bfloat16* g = (gate.has_value() && gate->defined()) ? reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr()) : nullptr;
  const int64_t warps = T * a.Hq;
  launch_pdl(attn_combine_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, st,
      a.part_o, a.part_ml, (int)T, a.Hq, a.nsplit, a.v_scale, g, g ? gate->stride(0) : 0,
      (out.has_value() && out->defined()) ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr,
      (out_q.has_value() && out_q->defined()) ? out_q->data_ptr<uint8_t>() : nullptr,
      (out_sf.has_value() && out_sf->defined()) ? out_sf->data_ptr<uint8_t>() : nullptr, (int)(a.Hq * fa::D / 32));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// prefill: one CTA per (query tile, kv head), output written directly (gate + MXFP8 fused)
void attn_tc_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                     torch::Tensor tok_ctx, torch::Tensor tile_tab, int64_t ntiles, double sm_scale, double k_scale,
                     double v_scale, c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> out,
                     c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_sf, torch::Tensor status) {
  if (ntiles == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  AttnArgs a = base_args(q, k_cache, block_table, tok_ctx, sm_scale, k_scale, v_scale, status);
  a.mode = 1;
  a.tile_tab = tile_tab.data_ptr<int32_t>();
  a.ntiles = (int)ntiles;
  if (gate.has_value() && gate->defined()) {
    a.gate = reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr());
    a.ld_gate = gate->stride(0);
  }
  a.out_bf16 = (out.has_value() && out->defined()) ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  a.out_q = (out_q.has_value() && out_q->defined()) ? out_q->data_ptr<uint8_t>() : nullptr;
  a.out_sf = (out_sf.has_value() && out_sf->defined()) ? out_sf->data_ptr<uint8_t>() : nullptr;
  a.out_kblocks = a.Hq * fa::D / 32;
  attn_tc_launch(a, kv_tmap(k_cache), kv_tmap(v_cache), dim3((unsigned)ntiles, (unsigned)a.Hkv, 1),
                 at::cuda::getCurrentCUDAStream());
}

}  // namespace r9k
