// tcgen05 GEMM core for sm_100a.
//
//   Y[tok, row] = sum_k W[row, k] * X[tok, k]      (weights are the MMA's A operand, tokens are B)
//
// One kernel template covers every linear layer of the framework:
//   * KIND_BF16: bf16 W x bf16 X, tcgen05.mma kind::f16.
//   * KIND_MX:   MXFP4 (e2m1) or MXFP8 (e4m3) W x MXFP8 X with ue8m0 block-32 scale factors in TMEM,
//                tcgen05.mma kind::mxf8f6f4.block_scale. NVFP4 and block-128 fp8 checkpoints are
//                converted to these at load (the reference does the same conversion on RDNA4:
//                r9700_vllm/quant/nvfp4.py:78, r9700_vllm/linear/fp8_block.py:23).
// Weights sit on the M side (128 rows per CTA), so a decode batch of 1..16 tokens is a single
// N=16 MMA ("swap-AB"), and prefill uses N=128/256 token tiles.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer,
// warps 2..5 = epilogue (TMEM -> registers -> global). Operand tiles arrive by TMA with the
// 128-byte swizzle; fp4 weights use the 16U4_ALIGN16B form the f8f6f4 MMA reads. Scale factors
// arrive as 512-byte bulk copies and go to TMEM with tcgen05.cp.
//
// Skinny (decode) GEMMs stream weights: fp4 weights are TMA-loaded packed (plain byte copies of
// contiguous 8 KB units, a deep ring) and the epilogue warps, idle during the main loop, expand each
// tile into the padded 16-element-group layout the f8f6f4 MMA reads -- the TMA's own fp4 expansion
// form streams at about half the rate. K is split so that two CTAs run per SM; each split parks its
// fp32 partial in a global workspace and the last split of a tile to arrive (per-tile counter, left
// at zero) sums the splits in split order (deterministic) and runs the epilogue.
//
// Epilogues: bf16 store (+ residual add, alpha), fp32 store, and the fused SwiGLU -> MXFP8 quant
// used by gate_up projections (two accumulators, gate and up, per CTA) that writes the down
// projection's input directly. Reference counterparts: kernels/r9k_moe_mxfp4a8.hip:187-480
// (FUSE=1 gate+up+silu), kernels/r9k_gemm_fp8.hip:36-222, kernels/r9k_moe_mxfp4a8.hip:811.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <map>
#include <mutex>
#include <tuple>
#include <unordered_map>
#include "gemm_common.cuh"

namespace r9k {

template <int KIND, int BN, bool DUAL, int NP, int NC, bool UNPACK, int MT = 1>
struct GemmCfg {
  static constexpr int NA = DUAL ? 2 : 1;
  static constexpr int A_BYTES = 128 * 128;                  // MMA-ready A tile (SW128)
  static constexpr int AL_BYTES = UNPACK ? 128 * 64 : A_BYTES;  // A as loaded (packed fp4 when UNPACK)
  static constexpr int B_BYTES = BN * 128;
  static constexpr int NB_SF = (BN + 127) / 128;
  static constexpr int SFA_BYTES = (KIND == KIND_MX) ? 512 : 0;
  static constexpr int SFB_BYTES = (KIND == KIND_MX) ? 512 * NB_SF : 0;
  // load ring (NP stages): A as loaded, B, scale factors
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + NP * NA * AL_BYTES;
  static constexpr int OFF_SFA = OFF_B + NP * B_BYTES;
  static constexpr int OFF_SFB = OFF_SFA + NP * NA * SFA_BYTES;
  // converted ring (NC stages, UNPACK only), 1 KiB aligned for the 128-byte swizzle
  static constexpr int OFF_C = (OFF_SFB + NP * SFB_BYTES + 1023) / 1024 * 1024;
  static constexpr int OFF_BAR = OFF_C + (UNPACK ? NC * NA * A_BYTES : 0);
  static constexpr int NUM_BARS = 2 * NP + 2 * NC + 1;
  static constexpr int OFF_TMEMPTR = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEMPTR + 16 + 1024;  // + alignment slack
  // TMEM columns: NACC independent accumulators (skinny tiles round-robin their K steps over them so
  // consecutive MMAs do not serialise on one accumulator), then scale factors
  static constexpr int NACC1 = BN == 16 ? 4 : BN == 32 ? (DUAL ? 2 : 4) : BN == 64 ? (DUAL ? 1 : 2) : 1;  // <= 256 TMEM cols (2 CTAs/SM)
  // MT row tiles per CTA (grouped skinny GEMMs): every tile keeps its own accumulators until the end
  static constexpr int NACC = MT == 1 ? NACC1 : (NACC1 >= 2 ? 2 : 1);
  static constexpr int ACC_TILE = BN * NA * NACC;  // TMEM columns of one row tile's accumulators
  static constexpr int ACC_COLS = ACC_TILE * MT;
  // scale factors: one TMEM set per load stage, so the tcgen05.cp of chunk q + 1 writes other columns
  // than the ones chunk q's MMAs still read and the two overlap in the tensor pipe
  static constexpr int SF_SETS = (KIND == KIND_MX) ? NP : 1;
  static constexpr int SF_STRIDE = 4 * NA + 4 * NB_SF;
  static constexpr int SFA_COL = ACC_COLS;
  static constexpr int SFB_COL = SFA_COL + 4 * NA;
  static constexpr int USED_COLS = (KIND == KIND_MX) ? ACC_COLS + SF_SETS * SF_STRIDE : ACC_COLS;
  static constexpr int TMEM_COLS = USED_COLS <= 32 ? 32 : USED_COLS <= 64 ? 64 : USED_COLS <= 128 ? 128
                                   : USED_COLS <= 256 ? 256 : 512;
  static constexpr int TILE_F = NA * BN * 128;  // floats of one split-K partial tile
  static_assert(!UNPACK || KIND == KIND_MX, "fp4 unpacking is for MX weights");
};

// Expand a packed e2m1 tile (128 rows x 64 B, row-major) into the 16U4_ALIGN16B form the f8f6f4 MMA
// reads (each 16-element group in the low 8 bytes of a 16-byte chunk), 128-byte swizzled.
// Thread t (0..127) converts row t.
R9K_DEVINL void unpack_fp4_tile(const uint8_t* src, uint8_t* dst, int r) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src + r * 64);
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int j = (jj + r) & 3;  // rotate to spread shared-memory banks
    const uint4 v = s4[j];
    const int c0 = 2 * j, c1 = 2 * j + 1;
    *reinterpret_cast<uint4*>(dst + r * 128 + ((c0 ^ (r & 7)) << 4)) = make_uint4(v.x, v.y, 0u, 0u);
    *reinterpret_cast<uint4*>(dst + r * 128 + ((c1 ^ (r & 7)) << 4)) = make_uint4(v.z, v.w, 0u, 0u);
  }
}

template <int KIND, int BN, bool DUAL, int EPI, int NP, int NC, bool UNPACK, int MT = 1>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB, const GemmArgs args, float* __restrict__ ws_part,
                   int* __restrict__ ws_cnt) {
  using C = GemmCfg<KIND, BN, DUAL, NP, NC, UNPACK, MT>;
  static_assert(MT == 1 || (!UNPACK && EPI != EPI_PUSH), "multi-tile CTAs: plain loads, local epilogues");
  constexpr int kPartStride = BN + 4;  // floats per parked row (cluster split-K): 16-byte rows, no bank conflicts
  static_assert(C::NA * 128 * kPartStride * 4 <= C::OFF_BAR, "parked partials fit in the idle operand ring");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* l_full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* l_empty = l_full + NP;
  uint64_t* c_full = l_empty + NP;
  uint64_t* c_empty = c_full + NC;
  uint64_t* tmem_full = c_empty + NC;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEMPTR);
  __shared__ int s_last, s_ok;

  const int warp = warp_id(), lane = lane_id();
  unsigned long long* tr =
      args.trace ? args.trace + ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * kTrN : nullptr;
  if (tr && threadIdx.x == 0) tr[kTrEntry] = globaltimer_ns();
  int m0 = blockIdx.x * 128 * MT;  // row (A) coordinate in the weight matrix (first of MT row tiles)
  const int S = args.splits;
  const int split = (int)(blockIdx.y % S);
  const int n_tile = (int)(blockIdx.y / S);
  int n0 = n_tile * BN;
  int m_valid = args.M;  // token rows [0, m_valid) are stored
  if (args.g_work != nullptr) {
    // grouped: the work list comes from the previous kernel
    pdl_wait();
    if ((int)blockIdx.y >= *args.g_count) return;
    const int e = args.g_work[3 * blockIdx.y + 0];
    n0 = args.g_work[3 * blockIdx.y + 1];
    m_valid = n0 + args.g_work[3 * blockIdx.y + 2];
    m0 = (e * args.g_row_tiles + (int)blockIdx.x * MT) * 128;
  }
  const int kc0 = split * args.kc_per_split;
  const int kc1 = min(args.kchunks, kc0 + args.kc_per_split);
  const int nk = max(0, kc1 - kc0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NP; ++i) {
      mbar_init(&l_full[i], 1);
      mbar_init(&l_empty[i], 1);
    }
    for (int i = 0; i < NC; ++i) {
      mbar_init(&c_full[i], 128);
      mbar_init(&c_empty[i], 1);
    }
    mbar_init(tmem_full, 1);
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (DUAL) prefetch_tmap(&tmA2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  if (tr && threadIdx.x == 0) tr[kTrSetup] = globaltimer_ns();

  const uint32_t a_tx = (KIND == KIND_BF16) ? 128 * 128 : (args.a_fmt == kFmtE2M1 ? 128 * 64 : 128 * 128);
  const uint32_t stage_tx = a_tx * C::NA + BN * 128 + (KIND == KIND_MX ? 512 * C::NA + 512 * C::NB_SF : 0);
  const int box_x = (KIND == KIND_BF16) ? 64 : (UNPACK ? 64 : 128);  // TMA box inner extent (elements of the map)
  const int kchunks_sf = (args.sf_kblocks + 3) / 4;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      // Weights do not depend on the previous kernel: the first NP weight tiles are requested before
      // waiting on the predecessor grid (programmatic dependent launch). Activations come after.
      // chunk q of this CTA: row tile q / nk, k-chunk q % nk (MT row tiles stream through one ring;
      // with MT == 1 both fold away at compile time)
      auto load_a = [&](int q) {
        const int s = q % NP;
        const int kc = kc0 + (MT == 1 ? q : q % nk);
        const int mt = m0 + (MT == 1 ? 0 : q / nk) * 128;
        uint8_t* sa = smem + C::OFF_A + s * C::NA * C::AL_BYTES;
        mbar_arrive_expect_tx(&l_full[s], stage_tx);
        load_a_tile(sa, &tmA, &l_full[s], args, kc, box_x, mt, pol_w);
        if (DUAL) load_a_tile(sa + C::AL_BYTES, &tmA2, &l_full[s], args, kc, box_x, mt, pol_w);
        if constexpr (KIND == KIND_MX) {
          uint8_t* ssfa = smem + C::OFF_SFA + s * C::NA * 512;
          bulk_load(ssfa, args.sfa + ((int64_t)(mt >> 7) * kchunks_sf + kc) * 512, 512, &l_full[s]);
          if (DUAL) bulk_load(ssfa + 512, args.sfa2 + ((int64_t)(mt >> 7) * kchunks_sf + kc) * 512, 512, &l_full[s]);
        }
      };
      auto load_b = [&](int q) {
        const int s = q % NP;
        const int kc = kc0 + (MT == 1 ? q : q % nk);
        tma_load_2d_hint(smem + C::OFF_B + s * C::B_BYTES, &tmB, &l_full[s], kc * ((KIND == KIND_BF16) ? 64 : 128), n0,
                         pol_x);
        if constexpr (KIND == KIND_MX) {
          uint8_t* ssfb = smem + C::OFF_SFB + s * C::SFB_BYTES;
#pragma unroll
          for (int c = 0; c < C::NB_SF; ++c)
            bulk_load(ssfb + 512 * c, args.sfb + ((int64_t)((n0 >> 7) + c) * kchunks_sf + kc) * 512, 512, &l_full[s]);
        }
      };
      // L2 prefetch of the weight chunk PD loads ahead of the ring: more bytes in flight than the
      // shared-memory stages alone hold (weights only; activations are small and L2-resident)
      const int PD = args.l2_prefetch;
      auto prefetch_a = [&](int q) {
        const int kc = kc0 + (MT == 1 ? q : q % nk);
        const int mt = m0 + (MT == 1 ? 0 : q / nk) * 128;
        prefetch_a_tile(&tmA, args, kc, box_x, mt);
        if (DUAL) prefetch_a_tile(&tmA2, args, kc, box_x, mt);
        if constexpr (KIND == KIND_MX) {
          bulk_prefetch_l2(args.sfa + ((int64_t)(mt >> 7) * kchunks_sf + kc) * 512, 512);
          if (DUAL) bulk_prefetch_l2(args.sfa2 + ((int64_t)(mt >> 7) * kchunks_sf + kc) * 512, 512);
        }
      };
      const int nq = nk * MT;
      const int npre = min(NP, nq);
      for (int q = 0; q < npre; ++q) load_a(q);
      for (int q = npre; q < min(nq, npre + PD); ++q) prefetch_a(q);
      pdl_wait();
      if (tr) tr[kTrPdl] = globaltimer_ns();
      for (int q = 0; q < nq; ++q) {
        if (q >= npre) {
          if (!mbar_wait(&l_empty[q % NP], (uint32_t)(((q / NP) & 1) ^ 1), args.timeout_ns)) {
            report_error(args.status, kErrMbarTimeout, 100, q);
            break;
          }
          load_a(q);
          if (PD > 0 && q + PD < nq) prefetch_a(q + PD);
        }
        load_b(q);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      for (int q = 0; q < nk * MT; ++q) {
        const int s = q % NP;
        const int sc = q % NC;
        const int i = MT == 1 ? q : q % nk;  // k-chunk within the row tile
        if (!mbar_wait(&l_full[s], (uint32_t)((q / NP) & 1), args.timeout_ns) ||
            (UNPACK && !mbar_wait(&c_full[sc], (uint32_t)((q / NC) & 1), args.timeout_ns))) {
          report_error(args.status, kErrMbarTimeout, 101, q);
          break;
        }
        if (tr && q == 0) tr[kTrFirst] = globaltimer_ns();
        tc_fence_after();
        const uint32_t sa = UNPACK ? smem_u32(smem + C::OFF_C + sc * C::NA * C::A_BYTES)
                                   : smem_u32(smem + C::OFF_A + s * C::NA * C::AL_BYTES);
        const uint32_t sb = smem_u32(smem + C::OFF_B + s * C::B_BYTES);
        const uint32_t sfo = (uint32_t)((q % C::SF_SETS) * C::SF_STRIDE);  // this stage's scale-factor set
        if constexpr (KIND == KIND_MX) {
          const uint32_t ssfa = smem_u32(smem + C::OFF_SFA + s * C::NA * 512);
          const uint32_t ssfb = smem_u32(smem + C::OFF_SFB + s * C::SFB_BYTES);
          tc_cp_32x128b_warpx4(tbase + C::SFA_COL + sfo, sdesc_sf(ssfa));
          if (DUAL) tc_cp_32x128b_warpx4(tbase + C::SFA_COL + sfo + 4, sdesc_sf(ssfa + 512));
#pragma unroll
          for (int c = 0; c < C::NB_SF; ++c)
            tc_cp_32x128b_warpx4(tbase + C::SFB_COL + sfo + 4 * c, sdesc_sf(ssfb + 512 * c));
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t bd = sdesc_k_sw128(sb + 32 * k);
          const int ai = k % C::NACC;
          const uint32_t dacc = tbase + (uint32_t)((MT == 1 ? 0 : q / nk) * C::ACC_TILE + ai * BN * C::NA);
          const uint32_t acc = (i > 0 || k >= C::NACC) ? 1u : 0u;
          if constexpr (KIND == KIND_MX) {
            const uint32_t idesc = idesc_block_scaled(args.a_fmt, kFmtE4M3, 128, BN, (uint32_t)k, (uint32_t)k);
            const uint32_t sfb_addr = (tbase + C::SFB_COL + sfo) | ((uint32_t)k << 30);
            mma_mxf8f6f4_ss(dacc, sdesc_k_sw128(sa + 32 * k), bd, idesc, acc,
                            (tbase + C::SFA_COL + sfo) | ((uint32_t)k << 30), sfb_addr);
            if (DUAL)
              mma_mxf8f6f4_ss(dacc + BN, sdesc_k_sw128(sa + C::A_BYTES + 32 * k), bd, idesc, acc,
                              (tbase + C::SFA_COL + sfo + 4) | ((uint32_t)k << 30), sfb_addr);
          } else {
            constexpr uint32_t idesc = idesc_dense(kFmtBF16, kFmtBF16, 128, BN);
            mma_f16_ss(dacc, sdesc_k_sw128(sa + 32 * k), bd, idesc, acc);
            if (DUAL) mma_f16_ss(dacc + BN, sdesc_k_sw128(sa + C::A_BYTES + 32 * k), bd, idesc, acc);
          }
        }
        tc_commit(&l_empty[s]);
        if (UNPACK) tc_commit(&c_empty[sc]);
      }
      tc_commit(tmem_full);  // arrives once every MMA issued above has completed
      if (tr) tr[kTrIssued] = globaltimer_ns();
      pdl_trigger();
    }
    __syncwarp();
  } else {
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_local = q * 32 + lane;
    const int ct = threadIdx.x - 64;  // 0..127
    // ------------------------------ fp4 expansion (UNPACK) ------------------------------
    if constexpr (UNPACK) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % NP, sc = i % NC;
        const bool w1 = mbar_wait(&l_full[s], (uint32_t)((i / NP) & 1), args.timeout_ns);
        const bool w2 = mbar_wait(&c_empty[sc], (uint32_t)(((i / NC) & 1) ^ 1), args.timeout_ns);
        if (!w1 || !w2) {
          report_error(args.status, kErrMbarTimeout, 103, i);
          break;
        }
        const uint8_t* src = smem + C::OFF_A + s * C::NA * C::AL_BYTES;
        uint8_t* dst = smem + C::OFF_C + sc * C::NA * C::A_BYTES;
        unpack_fp4_tile(src, dst, ct);
        if (DUAL) unpack_fp4_tile(src + C::AL_BYTES, dst + C::A_BYTES, ct);
        fence_proxy_async();
        mbar_arrive(&c_full[sc]);
      }
    }
    // ------------------------------ epilogue ------------------------------
    GemmArgs ea = args;  // grouped mode: rows are the expert's own, tokens end at m_valid
    ea.M = m_valid;
    const int row = (args.g_work != nullptr ? (int)blockIdx.x * 128 * MT : m0) + row_local;
    const uint32_t trow = tbase + ((uint32_t)(q * 32) << 16);
    pdl_wait();
    ArCall arc;
    if constexpr (EPI == EPI_PUSH) arc = ar_resolve(args.peers, args.ar_call);
    const bool wok = __all_sync(0xffffffffu, nk == 0 || mbar_wait(tmem_full, 0, args.timeout_ns));
    if (threadIdx.x == 64) s_ok = 1;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!wok && lane == 0) s_ok = 0;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const bool ok = s_ok != 0;
    if (!ok) report_error(args.status, kErrMbarTimeout, 102, 0);
    if (tr && threadIdx.x == 64) tr[kTrAcc] = globaltimer_ns();
    tc_fence_after();
    // load one 16-column chunk of the accumulator(s), summing the NACC partial accumulators
    auto load_acc_t = [&](int t, int c, float* g, float* u) {
      const uint32_t tr = trow + (uint32_t)(t * C::ACC_TILE);
      tmem_ld16(tr + c, g);
      if (DUAL) tmem_ld16(tr + BN + c, u);
      tmem_ld_wait();
#pragma unroll
      for (int ai = 1; ai < C::NACC; ++ai) {
        float g2[16], u2[16];
        tmem_ld16(tr + ai * BN * C::NA + c, g2);
        if (DUAL) tmem_ld16(tr + ai * BN * C::NA + BN + c, u2);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          g[t] += g2[t];
          if (DUAL) u[t] += u2[t];
        }
      }
    };
    auto load_acc = [&](int c, float* g, float* u) { load_acc_t(0, c, g, u); };
    // EPI_PUSH: the bf16 tile is staged in shared memory as [token][128 rows] (the operand buffers are
    // free once the accumulator is complete) and pushed to every rank's slot as 16-byte vectors, so
    // NVLink carries full 256-byte row segments; then one thread raises the tile's flags.
    __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem);
    auto stage_push = [&](int c, const float* g) {
#pragma unroll
      for (int t = 0; t < 16; ++t) stg[(c + t) * 128 + row_local] = __float2bfloat16(g[t] * args.alpha);
    };
    auto flush_push = [&]() {
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const uint4* src = reinterpret_cast<const uint4*>(stg);
      const int W = args.peers.world;
      if (args.ar_ll) {
        // LL slots: two bf16 + the epoch per 8-byte word, buffer call % 2 (see comm.cuh); the data is
        // its own ready signal, so no fence and no tile flag follow
        const uint32_t ep = ar_global_call(args.peers, args.ar_call) + 1u;
        const uint32_t lb = (uint32_t)args.ar_call & 1u;
        for (int idx = ct; idx < args.M * 16; idx += 128) {
          const int tok = idx >> 4, ch = idx & 15;
          const uint4 v = src[tok * 16 + ch];
          const int64_t off = (int64_t)tok * args.N + m0 + ch * 8;
#pragma unroll
          for (int p = 0; p < AR_MAX_WORLD; ++p) {
            if (p >= W) break;
            uint32_t* d = ar_ll_slot(args.peers, p, lb, args.peers.rank) + off;
            st_ll16(d, v.x, v.y, ep);
            st_ll16(d + 4, v.z, v.w, ep);
          }
        }
        return;
      }
      for (int idx = ct; idx < args.M * 16; idx += 128) {
        const int tok = idx >> 4, ch = idx & 15;
        const uint4 v = src[tok * 16 + ch];
        const int64_t off = (int64_t)tok * args.N + m0 + ch * 8;
#pragma unroll
        for (int p = 0; p < AR_MAX_WORLD; ++p)
          if (p < W) *reinterpret_cast<uint4*>(arc.dst[p] + off) = v;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) ar_raise_flags(args.peers, args.ar_call, blockIdx.x, arc.epoch);
    };
    (void)stage_push;
    (void)flush_push;
    if (S == 1) {
      if (ok && nk > 0) {
#pragma unroll 1
        for (int t = 0; t < MT; ++t) {
#pragma unroll 1
          for (int c = 0; c < BN; c += 16) {
            float g[16], u[16];
            load_acc_t(t, c, g, u);
            if constexpr (EPI == EPI_PUSH) stage_push(c, g);
            else epilogue_chunk<BN, DUAL, EPI>(ea, g, u, row + t * 128, n0 + c, lane, &arc);
          }
        }
      }
      if constexpr (EPI == EPI_PUSH) flush_push();
    } else if (args.cluster_k) {
      // cluster split-K: park this split's fp32 partial [NA][128 rows][BN + 4] in this CTA's shared
      // memory (the operand ring is idle once the accumulator is complete; a row's tokens are
      // contiguous, so the peers read them as 16-byte vectors); the splits meet below
      float* mypart = reinterpret_cast<float*>(smem);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float g[16], u[16];
        if (nk > 0 && ok) {
          load_acc(c, g, u);
        } else {
#pragma unroll
          for (int t = 0; t < 16; ++t) g[t] = u[t] = 0.f;
        }
        float4* pg = reinterpret_cast<float4*>(mypart + row_local * kPartStride + c);
        float4* pu = reinterpret_cast<float4*>(mypart + 128 * kPartStride + row_local * kPartStride + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          pg[j] = make_float4(g[4 * j], g[4 * j + 1], g[4 * j + 2], g[4 * j + 3]);
          if (DUAL) pu[j] = make_float4(u[4 * j], u[4 * j + 1], u[4 * j + 2], u[4 * j + 3]);
        }
      }
    } else if (ok) {
      // split-K: park the fp32 partial, the last split to arrive sums all splits in split order
      const int tile_id = n_tile * gridDim.x + blockIdx.x;
      float* mypart = ws_part + ((int64_t)tile_id * S + split) * C::TILE_F;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float g[16], u[16];
        if (nk > 0) {
          load_acc(c, g, u);
        } else {
#pragma unroll
          for (int t = 0; t < 16; ++t) g[t] = u[t] = 0.f;
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          mypart[(c + t) * 128 + row_local] = g[t];
          if (DUAL) mypart[BN * 128 + (c + t) * 128 + row_local] = u[t];
        }
      }
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        const int old = atomicAdd(&ws_cnt[tile_id], 1);
        s_last = (old == S - 1) ? 1 : 0;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (s_last) {
        __threadfence();
        const float* base = ws_part + (int64_t)tile_id * S * C::TILE_F;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float g[16], u[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) g[t] = u[t] = 0.f;
          // (unrolled so several splits' loads are in flight together; the sum stays in split order)
#pragma unroll 2
          for (int r = 0; r < S; ++r) {
            const float* src = base + (int64_t)r * C::TILE_F;
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              g[t] += __ldcg(src + (c + t) * 128 + row_local);
              if (DUAL) u[t] += __ldcg(src + BN * 128 + (c + t) * 128 + row_local);
            }
          }
          if constexpr (EPI == EPI_PUSH) stage_push(c, g);
          else epilogue_chunk<BN, DUAL, EPI>(ea, g, u, row, n0 + c, lane, &arc);
        }
        if constexpr (EPI == EPI_PUSH) flush_push();
        if (threadIdx.x == 64) ws_cnt[tile_id] = 0;
      }
    }
  }

  if (S > 1 && args.cluster_k) {
    // every split of the tile parked its partial; CTA r of the cluster owns the contiguous token slice
    // [r BN / S, (r + 1) BN / S) of the tile: for each 4-token group it needs, it requests the group
    // from all S splits at once (16-byte distributed-shared-memory loads, all in flight together),
    // then sums them in split order (deterministic) and runs the epilogue for its tokens
    if (tr && threadIdx.x == 64) tr[kTrParked] = globaltimer_ns();
    cluster_sync();
    if (tr && threadIdx.x == 64) tr[kTrSync1] = globaltimer_ns();
    if (warp >= 2) {
      const int row_local = (warp & 3) * 32 + lane;
      const uint32_t me = cluster_ctarank();
      const uint32_t my_base = smem_u32(smem);
      GemmArgs ea = args;
      ea.M = m_valid;
      const int tpc = BN / S;
      const int ta = (int)me * tpc, tb = ta + tpc;
#pragma unroll 1
      for (int c = ta & ~15; c < tb; c += 16) {
        uint32_t tmask = 0;
#pragma unroll
        for (int t = 0; t < 16; ++t)
          if (c + t >= ta && c + t < tb && n0 + c + t < m_valid) tmask |= 1u << t;
        if (tmask == 0) continue;
        float g[16], u[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) g[t] = u[t] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (((tmask >> (4 * j)) & 0xFu) == 0) continue;
          const uint32_t off = (uint32_t)((row_local * kPartStride + c + 4 * j) * 4);
          constexpr int KB = DUAL ? 2 : 4;  // splits requested per batch (bounded registers)
#pragma unroll 1
          for (int k0 = 0; k0 < S; k0 += KB) {
            float4 vg[KB], vu[KB];
#pragma unroll
            for (int k = 0; k < KB; ++k) {
              if (k0 + k < S) {
                const uint32_t rb = mapa_shared(my_base, (uint32_t)(k0 + k)) + off;
                vg[k] = ld_dsmem_v4(rb);
                if (DUAL) vu[k] = ld_dsmem_v4(rb + 128u * kPartStride * 4u);
              }
            }
#pragma unroll
            for (int k = 0; k < KB; ++k) {
              if (k0 + k < S) {
                g[4 * j] += vg[k].x; g[4 * j + 1] += vg[k].y; g[4 * j + 2] += vg[k].z; g[4 * j + 3] += vg[k].w;
                if (DUAL) {
                  u[4 * j] += vu[k].x; u[4 * j + 1] += vu[k].y; u[4 * j + 2] += vu[k].z; u[4 * j + 3] += vu[k].w;
                }
              }
            }
          }
        }
        epilogue_chunk<BN, DUAL, EPI>(ea, g, u, m0 + row_local, n0 + c, lane, nullptr, tmask);
      }
    }
    if (tr && threadIdx.x == 64) tr[kTrReduced] = globaltimer_ns();
    cluster_sync();  // no CTA leaves while a peer may still read its partial
    if (tr && threadIdx.x == 64) tr[kTrSync2] = globaltimer_ns();
  }

  tc_fence_before();
  __syncthreads();
  if (tr && threadIdx.x == 64) tr[kTrDone] = globaltimer_ns();
  if (tr && threadIdx.x == 0) tr[kTrDone0] = globaltimer_ns();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
template <int KIND, bool DUAL, int EPI>
bool gemm_sk_dispatch(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, const GemmArgs& a,
                      torch::Tensor& ws, cudaStream_t st);

struct LaunchPlan {
  int BN;
  int S;        // K splits
  int n_tiles;
  bool unpack;  // fp4 weights loaded packed and expanded on chip
};

static int num_sms() { return device_sm_count(); }

static bool gemm_cluster_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("R9K_GEMM_CLUSTER");
    v = (e && (e[0] == '0' || e[0] == 's')) ? 0 : 1;  // "0" / "stock": global-workspace split-K fix-up
  }
  return v == 1;
}

static LaunchPlan plan_gemm(int N, int M, int kchunks, bool dual, bool fp4) {
  LaunchPlan p;
  if (M <= 16) p.BN = 16;
  else if (M <= 32) p.BN = 32;
  else if (M <= 64) p.BN = 64;
  else if (M <= 128) p.BN = 128;
  else p.BN = dual ? 128 : 256;  // two accumulators of 256 columns would not fit in TMEM
  if (p.BN == 256 && M > 256) {
    const int rt = (N + 127) / 128;
    if ((long)rt * ((M + 255) / 256) < num_sms()) p.BN = 128;
  }
  static int force_bn = -1;
  if (force_bn < 0) {
    const char* e = getenv("R9K_GEMM_BN");  // tuning: force the token tile of prefill-sized GEMMs
    force_bn = e ? std::max(0, atoi(e)) : 0;
  }
  if (force_bn > 0 && M > 128 && (force_bn == 128 || (force_bn == 256 && !dual))) p.BN = force_bn;
  p.n_tiles = (M + p.BN - 1) / p.BN;
  static int unpack_knob = -1;
  if (unpack_knob < 0) {
    const char* e = getenv("R9K_FP4_UNPACK");
    unpack_knob = (e && e[0] == '1') ? 1 : 0;
  }
  p.unpack = unpack_knob == 1 && fp4 && p.BN <= 64;
  const int row_tiles = (N + 127) / 128;
  const int tiles = row_tiles * p.n_tiles;
  p.S = 1;
  if (p.BN <= 64) {
    // fill the resident CTA slots: split K (global-memory fix-up, no clusters) with >= 4 chunks/split
    const int per_sm = (dual && p.unpack) ? 1 : 2;
    const int target = per_sm * num_sms();
    // (at most 8 splits when they form a cluster: the portable cluster size)
    p.S = std::max(1, std::min(gemm_cluster_enabled() ? 8 : 16, target / std::max(1, tiles)));
    while (p.S > 1 && kchunks / p.S < 4) --p.S;
    static int force_s = -1;
    if (force_s < 0) {
      const char* e = getenv("R9K_GEMM_SPLITS");  // tuning: force the K split count of skinny GEMMs
      force_s = e ? std::max(0, atoi(e)) : 0;
    }
    if (force_s > 0) p.S = std::min(force_s, std::max(1, kchunks));
  }
  return p;
}

// tuning trace buffer (gemm_trace): the tiled kernel stamps kTrN timestamps per CTA when it fits
static unsigned long long* g_trace = nullptr;
static int64_t g_trace_cap = 0;

void gemm_trace(c10::optional<torch::Tensor> buf) {
  if (buf.has_value() && buf->defined()) {
    TORCH_CHECK(buf->is_cuda() && buf->dtype() == torch::kInt64 && buf->is_contiguous(), "gemm_trace: int64 cuda buffer");
    g_trace = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
    g_trace_cap = buf->numel();
  } else {
    g_trace = nullptr;
    g_trace_cap = 0;
  }
}

// workspace layout: [65536 int counters][partials]
static constexpr int64_t kWsCounters = 65536;

template <int KIND, int BN, bool DUAL, int EPI, int NP, int NC, bool UNPACK, int MT = 1>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, GemmArgs args,
                        LaunchPlan p, torch::Tensor* ws, cudaStream_t stream) {
  using C = GemmCfg<KIND, BN, DUAL, NP, NC, UNPACK, MT>;
  auto kern = gemm_tc_kernel<KIND, BN, DUAL, EPI, NP, NC, UNPACK, MT>;
  TORCH_CHECK(ensure_smem_attr((const void*)kern, C::SMEM_BYTES) == cudaSuccess, "r9k gemm: cannot set smem size");
  TORCH_CHECK(((args.N + 127) / 128) % MT == 0, "r9k gemm: row tiles must divide over the CTAs");
  const int grid_x = (args.N + 127) / 128 / MT;
  if (MT > 1) p.S = 1;  // multi-tile CTAs keep whole K
  float* part = nullptr;
  int* cnt = nullptr;
  if (p.S > 1) {
    const int64_t need = (int64_t)grid_x * p.n_tiles * p.S * C::TILE_F;
    if (ws == nullptr || ws->numel() < kWsCounters + need || grid_x * p.n_tiles > kWsCounters) p.S = 1;
    else {
      cnt = reinterpret_cast<int*>(ws->data_ptr<float>());
      part = ws->data_ptr<float>() + kWsCounters;
    }
  }
  // split-K partials meet in distributed shared memory when the splits of a tile form a cluster of 2,
  // 4 or 8 CTAs (measured: 7-CTA clusters of the 5120 x 17408 decode GEMM pack into fewer resident
  // clusters per GPC and take two waves, 27.6 vs 14.8 us; power-of-two clusters run faster than the
  // global fix-up, e.g. 2176 x 5120 gate/up 16.6 -> 12.3 us)
  const bool cluster = (p.S == 2 || p.S == 4 || p.S == 8) && EPI != EPI_PUSH && MT == 1 && gemm_cluster_enabled();
  if (cluster) {
    part = nullptr;
    cnt = nullptr;
  }
  args.cluster_k = cluster ? 1 : 0;
  args.splits = p.S;
  args.kc_per_split = (args.kchunks + p.S - 1) / p.S;
  static int l2pf = -1;
  if (l2pf < 0) {
    const char* e = getenv("R9K_GEMM_L2PF");
    l2pf = e ? std::max(0, atoi(e)) : 0;
  }
  if (BN <= 64 && !UNPACK) args.l2_prefetch = l2pf;  // skinny (weight-streaming) GEMMs only
  args.trace = ((int64_t)grid_x * p.n_tiles * p.S * kTrN <= g_trace_cap) ? g_trace : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid_x, p.n_tiles * p.S, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = cluster ? (unsigned)p.S : 1u;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, ta2, tb, args, part, cnt);
  TORCH_CHECK(e == cudaSuccess, "r9k gemm launch failed: ", cudaGetErrorString(e));
}

template <int KIND, bool DUAL, int EPI>
static void dispatch_bn(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, GemmArgs args,
                        const LaunchPlan& p, torch::Tensor* ws, cudaStream_t st) {
  // skinny tiles: two CTAs/SM (~110 KB each), fp4 expanded on chip with a deep packed ring;
  // wide tiles: one CTA/SM
  if constexpr (KIND == KIND_MX) {
    if (p.unpack) {
      switch (p.BN) {
        case 16: DUAL ? launch_gemm<KIND, 16, DUAL, EPI, 7, 2, true>(ta, ta2, tb, args, p, ws, st)
                      : launch_gemm<KIND, 16, DUAL, EPI, 6, 2, true>(ta, ta2, tb, args, p, ws, st); return;
        case 32: DUAL ? launch_gemm<KIND, 32, DUAL, EPI, 6, 2, true>(ta, ta2, tb, args, p, ws, st)
                      : launch_gemm<KIND, 32, DUAL, EPI, 5, 2, true>(ta, ta2, tb, args, p, ws, st); return;
        default: DUAL ? launch_gemm<KIND, 64, DUAL, EPI, 5, 2, true>(ta, ta2, tb, args, p, ws, st)
                      : launch_gemm<KIND, 64, DUAL, EPI, 4, 2, true>(ta, ta2, tb, args, p, ws, st); return;
      }
    }
  }
  switch (p.BN) {
    case 16: launch_gemm<KIND, 16, DUAL, EPI, DUAL ? 3 : 5, 1, false>(ta, ta2, tb, args, p, ws, st); break;
    case 32: launch_gemm<KIND, 32, DUAL, EPI, DUAL ? 3 : 5, 1, false>(ta, ta2, tb, args, p, ws, st); break;
    case 64: launch_gemm<KIND, 64, DUAL, EPI, DUAL ? 2 : 4, 1, false>(ta, ta2, tb, args, p, ws, st); break;
    case 128: launch_gemm<KIND, 128, DUAL, EPI, DUAL ? 3 : 4, 1, false>(ta, ta2, tb, args, p, ws, st); break;
    default:
      if constexpr (!DUAL) launch_gemm<KIND, 256, false, EPI, 4, 1, false>(ta, ta2, tb, args, p, ws, st);
      break;
  }
}

// activation scale buffers must cover every token tile the kernel touches (rows rounded up to BN)
static void check_act_sf(const torch::Tensor& sf, const LaunchPlan& p, int64_t K, const char* what) {
  const int64_t rows = (int64_t)p.n_tiles * p.BN;
  const int64_t need = ((rows + 127) / 128) * ((K / 32 + 3) / 4) * 512;
  TORCH_CHECK(sf.numel() >= need, what, ": activation scales must cover ", rows, " rows (allocate rows rounded up to 256)");
}

static void check_sf(const torch::Tensor& sf, int64_t rows, int64_t K, const char* what) {
  const int64_t need = ((rows + 127) / 128) * ((K / 32 + 3) / 4) * 512;
  TORCH_CHECK(sf.dtype() == torch::kUInt8 && sf.is_contiguous(), what, ": scale tensor must be contiguous uint8");
  TORCH_CHECK(sf.numel() >= need, what, ": scale tensor too small (", sf.numel(), " < ", need, ")");
}

// out[M, N] = X[M, K] @ W[N, K]^T with MX formats.
//   w: uint8 [N, K/2] (fp4, w_fp4=true) or [N, K] (e4m3); w_sf: chunk-layout ue8m0
//   x: uint8 [M, K] e4m3; x_sf: chunk-layout ue8m0
//   epi: 0 bf16 (+residual), 1 f32
// weights: [N, K/2 | K] row-major, or pre-tiled [units, 128, 64 | 128] (units = ceil(N/128) * K/128)
static CUtensorMap weight_tmap(const torch::Tensor& w, bool fp4, int64_t N, int64_t K, bool unpack) {
  if (w.dim() == 3) {
    TORCH_CHECK(w.size(1) == 128 && w.size(2) == (fp4 ? 64 : 128) && w.is_contiguous(), "tiled weight shape");
    TORCH_CHECK(w.size(0) == ((N + 127) / 128) * (K / 128), "tiled weight: unit count does not match N, K");
    if (unpack) return tmap_units_packed_3d(w.data_ptr(), w.size(0));
    return tmap_units_3d(w.data_ptr(), w.size(0), fp4);
  }
  TORCH_CHECK(w.size(0) == N && w.size(1) == (fp4 ? K / 2 : K), "weight/activation shape mismatch");
  if (unpack) return tmap_fp4_packed(w.data_ptr(), N, K);
  return fp4 ? tmap_fp4_kmajor(w.data_ptr(), N, K, 128) : tmap_u8_kmajor(w.data_ptr(), N, K, 128);
}

bool gemm_mx_swap(const CUtensorMap& tw, const torch::Tensor& x, const torch::Tensor& x_sf, const torch::Tensor& w_sf,
                  bool w_fp4, bool w_tiled, torch::Tensor& out, const c10::optional<torch::Tensor>& residual, double alpha,
                  torch::Tensor& status);

bool gemm_bf16_swap(const torch::Tensor& w, const torch::Tensor& x, torch::Tensor& out,
                    const c10::optional<torch::Tensor>& residual, double alpha, torch::Tensor& status);

static bool gemm_swap_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("R9K_GEMM_SWAP");
    v = (e && (e[0] == '0' || e[0] == 's')) ? 0 : 1;  // "0" / "stock": weight rows on the MMA's M side
  }
  return v == 1;
}

static bool use_stream_k() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("R9K_GEMM_SK");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

void gemm_mx(torch::Tensor w, torch::Tensor w_sf, bool w_fp4, torch::Tensor x, torch::Tensor x_sf,
             torch::Tensor out, c10::optional<torch::Tensor> residual, double alpha, torch::Tensor status,
             c10::optional<torch::Tensor> workspace) {
  const int64_t N = out.size(1), M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0, "gemm_mx: K must be a multiple of 128");
  check_sf(w_sf, N, K, "gemm_mx weight");
  check_sf(x_sf, M, K, "gemm_mx activation");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "gemm_mx: bad out");
  const bool f32 = out.dtype() == torch::kFloat32;
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  LaunchPlan p = plan_gemm((int)N, (int)M, (int)(K / 128), false, w_fp4);
  check_act_sf(x_sf, p, K, "gemm_mx");
  const bool sk = use_stream_k() && M <= 64;
  if (sk) p.unpack = false;
  CUtensorMap ta = weight_tmap(w, w_fp4, N, K, p.unpack);
  CUtensorMap tb = tmap_u8_kmajor(x.data_ptr(), M, K, p.BN);
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 128);
  a.a_fmt = w_fp4 ? kFmtE2M1 : kFmtE4M3;
  a.a_tiled = w.dim() == 3;
  a.sfa = w_sf.data_ptr<uint8_t>(); a.sfb = x_sf.data_ptr<uint8_t>(); a.sf_kblocks = (int)(K / 32);
  a.out = out.data_ptr(); a.ldo = (int)out.stride(0);
  if (residual.has_value() && residual->defined()) {
    TORCH_CHECK(!f32, "residual add needs bf16 output");
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ldr = (int)residual->stride(0);
  }
  a.alpha = (float)alpha;
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
  auto st = at::cuda::getCurrentCUDAStream();
  torch::Tensor* ws = (workspace.has_value() && workspace->defined()) ? &(*workspace) : nullptr;
  if (sk && ws != nullptr) {
    const bool done = f32 ? gemm_sk_dispatch<KIND_MX, false, EPI_F32>(ta, ta, tb, a, *ws, st)
                          : gemm_sk_dispatch<KIND_MX, false, EPI_BF16>(ta, ta, tb, a, *ws, st);
    if (done) return;
    p = plan_gemm((int)N, (int)M, (int)(K / 128), false, w_fp4);
    ta = weight_tmap(w, w_fp4, N, K, p.unpack);
  }
  if (p.BN >= 128 && M >= 256 && !p.unpack && gemm_swap_enabled() &&
      gemm_mx_swap(ta, x, x_sf, w_sf, w_fp4, w.dim() == 3, out, residual, alpha, status))
    return;  // prefill-sized M: tokens on the MMA's M side, vector epilogue (gemm_swap.cu)
  if (f32) dispatch_bn<KIND_MX, false, EPI_F32>(ta, ta, tb, a, p, ws, st);
  else dispatch_bn<KIND_MX, false, EPI_BF16>(ta, ta, tb, a, p, ws, st);
}

// Row-parallel GEMM whose epilogue performs the all-reduce's communication: the bf16 result tile is
// stored into slot [rank] of every rank's symmetric region and the tile's flag is raised; ar_rmsnorm
// on each rank then reduces. Decode-sized batches only (one token tile).
void gemm_mx_push(torch::Tensor w, torch::Tensor w_sf, bool w_fp4, torch::Tensor x, torch::Tensor x_sf, int64_t N,
                  torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call, torch::Tensor step,
                  int64_t calls_per_step, torch::Tensor status, c10::optional<torch::Tensor> workspace, int64_t ll) {
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0, "gemm_mx_push: K and N multiples of 128");
  TORCH_CHECK(M * N <= slot_elems, "gemm_mx_push: output exceeds the slot");
  check_sf(w_sf, N, K, "gemm_mx_push weight");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  LaunchPlan p = plan_gemm((int)N, (int)M, (int)(K / 128), false, w_fp4);
  TORCH_CHECK(p.n_tiles == 1, "gemm_mx_push: at most one token tile (<= 256 tokens)");
  check_act_sf(x_sf, p, K, "gemm_mx_push");
  CUtensorMap ta = weight_tmap(w, w_fp4, N, K, p.unpack);
  CUtensorMap tb = tmap_u8_kmajor(x.data_ptr(), M, K, p.BN);
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 128);
  a.a_fmt = w_fp4 ? kFmtE2M1 : kFmtE4M3;
  a.a_tiled = w.dim() == 3;
  a.sfa = w_sf.data_ptr<uint8_t>(); a.sfb = x_sf.data_ptr<uint8_t>(); a.sf_kblocks = (int)(K / 32);
  a.alpha = 1.f;
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
  a.peers = make_peers(peers, rank, world, slot_elems, N, step, calls_per_step);
  a.ar_call = (int)call;
  a.ar_ll = ll ? 1 : 0;
  torch::Tensor* ws = (workspace.has_value() && workspace->defined()) ? &(*workspace) : nullptr;
  dispatch_bn<KIND_MX, false, EPI_PUSH>(ta, ta, tb, a, p, ws, at::cuda::getCurrentCUDAStream());
}

// Grouped expert GEMM over expert-sorted token rows (see moe.cu). w / w_sf: stacked experts
// [E * N, K] (pre-tiled units); with w2 the gate/up pair runs with the SwiGLU -> MXFP8 epilogue,
// otherwise the bf16 result goes to out. Rows are processed in the BN-row tiles of the work list.
void gemm_mx_grouped(torch::Tensor w, torch::Tensor w_sf, c10::optional<torch::Tensor> w2,
                     c10::optional<torch::Tensor> w2_sf, bool w_fp4, torch::Tensor x, torch::Tensor x_sf,
                     torch::Tensor work, torch::Tensor work_count, int64_t N, int64_t E, int64_t BN, torch::Tensor out,
                     c10::optional<torch::Tensor> out_sf, torch::Tensor status) {
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0, "gemm_mx_grouped: K and N multiples of 128");
  const bool dual = w2.has_value() && w2->defined();
  const at::cuda::CUDAGuard guard(x.device());
  LaunchPlan p;
  p.BN = (int)BN;
  p.S = 1;
  p.n_tiles = (int)work.size(0);
  p.unpack = false;
  TORCH_CHECK(!(dual && BN > 128), "gemm_mx_grouped: dual needs BN <= 128");
  CUtensorMap ta = weight_tmap(w, w_fp4, E * N, K, false);
  CUtensorMap ta2 = dual ? weight_tmap(*w2, w_fp4, E * N, K, false) : ta;
  CUtensorMap tb = tmap_u8_kmajor(x.data_ptr(), M, K, p.BN);
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 128);
  a.a_fmt = w_fp4 ? kFmtE2M1 : kFmtE4M3;
  a.a_tiled = w.dim() == 3;
  a.sfa = w_sf.data_ptr<uint8_t>(); a.sfb = x_sf.data_ptr<uint8_t>(); a.sf_kblocks = (int)(K / 32);
  if (dual) a.sfa2 = w2_sf->data_ptr<uint8_t>();
  a.out = out.data_ptr(); a.ldo = (int)out.stride(0);
  if (dual) { a.out_sf = out_sf->data_ptr<uint8_t>(); a.out_kblocks = (int)(N / 32); }
  a.alpha = 1.f;
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
  a.g_work = work.data_ptr<int32_t>();
  a.g_count = work_count.data_ptr<int32_t>();
  a.g_row_tiles = (int)(N / 128);
  // grid.x = N / 128 row tiles of one expert; grid.y = work items (the launcher multiplies by S = 1)
  auto st = at::cuda::getCurrentCUDAStream();
  a.N = (int)N;
  GemmArgs ga = a;
  ga.N = (int)N;
  // launch_gemm derives grid.x from args.N. Skinny batches: several row tiles of an expert per CTA
  // (gate/up 2, down 4), so each CTA streams enough weight chunks to amortise its start-up and fill
  static int mt_knob = -1;
  if (mt_knob < 0) {
    const char* e = getenv("R9K_MOE_MT");
    mt_knob = (e && e[0] == '0') ? 0 : 1;
  }
  const int rt = (int)(N / 128);
  if (mt_knob && BN == 16 && dual && rt % 2 == 0) {
    launch_gemm<KIND_MX, 16, true, EPI_SWIGLU_MXFP8, 3, 1, false, 2>(ta, ta2, tb, ga, p, nullptr, st);
  } else if (mt_knob && BN == 16 && !dual && rt % 4 == 0) {
    launch_gemm<KIND_MX, 16, false, EPI_BF16, 5, 1, false, 4>(ta, ta, tb, ga, p, nullptr, st);
  } else if (dual) {
    dispatch_bn<KIND_MX, true, EPI_SWIGLU_MXFP8>(ta, ta2, tb, ga, p, nullptr, st);
  } else {
    dispatch_bn<KIND_MX, false, EPI_BF16>(ta, ta, tb, ga, p, nullptr, st);
  }
}

// Fused gate/up projection + SwiGLU + MXFP8 quantisation of the result.
void gemm_mx_swiglu(torch::Tensor wg, torch::Tensor wg_sf, torch::Tensor wu, torch::Tensor wu_sf, bool w_fp4,
                    torch::Tensor x, torch::Tensor x_sf, torch::Tensor out_q, torch::Tensor out_sf,
                    torch::Tensor status, c10::optional<torch::Tensor> workspace) {
  const int64_t N = out_q.size(1), M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0 && N % 32 == 0, "gemm_mx_swiglu: K % 128 and N % 32 required");
  TORCH_CHECK(wu.sizes() == wg.sizes(), "gemm_mx_swiglu: gate/up mismatch");
  check_sf(wg_sf, N, K, "swiglu gate");
  check_sf(wu_sf, N, K, "swiglu up");
  check_sf(x_sf, M, K, "swiglu act");
  check_sf(out_sf, M, N, "swiglu out");
  TORCH_CHECK(out_q.size(0) == M && out_q.size(1) == N, "gemm_mx_swiglu: bad out");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  LaunchPlan p = plan_gemm((int)N, (int)M, (int)(K / 128), true, w_fp4);
  check_act_sf(x_sf, p, K, "gemm_mx_swiglu");
  const bool sk = use_stream_k() && M <= 64;
  if (sk) p.unpack = false;
  CUtensorMap ta = weight_tmap(wg, w_fp4, N, K, p.unpack);
  CUtensorMap ta2 = weight_tmap(wu, w_fp4, N, K, p.unpack);
  CUtensorMap tb = tmap_u8_kmajor(x.data_ptr(), M, K, p.BN);
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 128);
  a.a_fmt = w_fp4 ? kFmtE2M1 : kFmtE4M3;
  a.a_tiled = wg.dim() == 3;
  a.sfa = wg_sf.data_ptr<uint8_t>(); a.sfa2 = wu_sf.data_ptr<uint8_t>(); a.sfb = x_sf.data_ptr<uint8_t>();
  a.sf_kblocks = (int)(K / 32);
  a.out = out_q.data_ptr(); a.ldo = (int)out_q.stride(0);
  a.out_sf = out_sf.data_ptr<uint8_t>(); a.out_kblocks = (int)(N / 32);
  a.alpha = 1.f;
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
  auto st = at::cuda::getCurrentCUDAStream();
  torch::Tensor* ws = (workspace.has_value() && workspace->defined()) ? &(*workspace) : nullptr;
  if (sk && ws != nullptr) {
    if (gemm_sk_dispatch<KIND_MX, true, EPI_SWIGLU_MXFP8>(ta, ta2, tb, a, *ws, st)) return;
    p = plan_gemm((int)N, (int)M, (int)(K / 128), true, w_fp4);
    ta = weight_tmap(wg, w_fp4, N, K, p.unpack);
    ta2 = weight_tmap(wu, w_fp4, N, K, p.unpack);
  }
  dispatch_bn<KIND_MX, true, EPI_SWIGLU_MXFP8>(ta, ta2, tb, a, p, ws, st);
}

// bf16 gate/up projection with the SwiGLU epilogue (bf16 result): dense bf16 FFNs and shared experts.
void gemm_bf16_swiglu(torch::Tensor wg, torch::Tensor wu, torch::Tensor x, torch::Tensor out, torch::Tensor status,
                      c10::optional<torch::Tensor> workspace) {
  const int64_t N = wg.size(0), M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 64 == 0 && wg.sizes() == wu.sizes() && wg.size(1) == K, "gemm_bf16_swiglu: shapes");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  LaunchPlan p = plan_gemm((int)N, (int)M, (int)(K / 64), true, false);
  CUtensorMap ta = tmap_bf16_kmajor(wg.data_ptr(), N, K, wg.stride(0), 128);
  CUtensorMap ta2 = tmap_bf16_kmajor(wu.data_ptr(), N, K, wu.stride(0), 128);
  CUtensorMap tb = tmap_bf16_kmajor(x.data_ptr(), M, K, x.stride(0), p.BN);
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 64);
  a.out = out.data_ptr(); a.ldo = (int)out.stride(0);
  a.alpha = 1.f;
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
  torch::Tensor* ws = (workspace.has_value() && workspace->defined()) ? &(*workspace) : nullptr;
  dispatch_bn<KIND_BF16, true, EPI_SWIGLU_BF16>(ta, ta2, tb, a, p, ws, at::cuda::getCurrentCUDAStream());
}

// bf16 x bf16 -> bf16/f32 (kind::f16)
void gemm_bf16(torch::Tensor w, torch::Tensor x, torch::Tensor out, c10::optional<torch::Tensor> residual,
               double alpha, torch::Tensor status, c10::optional<torch::Tensor> workspace) {
  const int64_t N = w.size(0), M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 64 == 0 && w.size(1) == K, "gemm_bf16: K must match and be a multiple of 64");
  TORCH_CHECK(w.dtype() == torch::kBFloat16 && x.dtype() == torch::kBFloat16, "gemm_bf16: bf16 inputs");
  TORCH_CHECK(w.stride(1) == 1 && x.stride(1) == 1, "gemm_bf16: inner stride 1");
  const bool f32 = out.dtype() == torch::kFloat32;
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  LaunchPlan p = plan_gemm((int)N, (int)M, (int)(K / 64), false, false);
  CUtensorMap ta = tmap_bf16_kmajor(w.data_ptr(), N, K, w.stride(0), 128);
  CUtensorMap tb = tmap_bf16_kmajor(x.data_ptr(), M, K, x.stride(0), p.BN);
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 64);
  a.out = out.data_ptr(); a.ldo = (int)out.stride(0);
  if (residual.has_value() && residual->defined()) {
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ldr = (int)residual->stride(0);
  }
  a.alpha = (float)alpha;
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
  auto st = at::cuda::getCurrentCUDAStream();
  torch::Tensor* ws = (workspace.has_value() && workspace->defined()) ? &(*workspace) : nullptr;
  if (use_stream_k() && M <= 64 && ws != nullptr) {
    const bool done = f32 ? gemm_sk_dispatch<KIND_BF16, false, EPI_F32>(ta, ta, tb, a, *ws, st)
                          : gemm_sk_dispatch<KIND_BF16, false, EPI_BF16>(ta, ta, tb, a, *ws, st);
    if (done) return;
  }
  if (p.BN >= 128 && M >= 256 && gemm_swap_enabled() && gemm_bf16_swap(w, x, out, residual, alpha, status))
    return;  // prefill-sized M: tokens on the MMA's M side (gemm_swap.cu)
  if (f32) dispatch_bn<KIND_BF16, false, EPI_F32>(ta, ta, tb, a, p, ws, st);
  else dispatch_bn<KIND_BF16, false, EPI_BF16>(ta, ta, tb, a, p, ws, st);
}

}  // namespace r9k

// ---------------------------------------------------------------------------------------------
// r9k_gemm_bf16_noalloc: the skinny bf16 GEMM with split-K scratch in a fixed device array (no
// allocation of any kind; declared and documented in r9k_noalloc.h).
// ---------------------------------------------------------------------------------------------
#include <cstdio>
#include <atomic>
#include "r9k_noalloc.h"

namespace {

constexpr int64_t kNaCounterInts = 1024;  // 4 KiB of per-tile counters
constexpr int64_t kNaPartFloats = (int64_t)(R9K_NOALLOC_SCRATCH_BYTES / 4) - kNaCounterInts;
constexpr int kNaMaxDev = 64;

__device__ __align__(256) float r9k_noalloc_scratch[R9K_NOALLOC_SCRATCH_BYTES / 4];

struct NaDevice {
  std::atomic<bool> ready{false};  // release-stored after scratch is set; acquire-loaded on the fast path
  float* scratch = nullptr;        // device address of r9k_noalloc_scratch on this device
};
NaDevice g_na[kNaMaxDev];
std::mutex g_na_mu;
r9k::EncodeTiledFn g_na_encode = nullptr;

template <int BN, int NP>
cudaError_t na_set_attr() {
  using C = r9k::GemmCfg<r9k::KIND_BF16, BN, false, NP, 1, false>;
  return cudaFuncSetAttribute(r9k::gemm_tc_kernel<r9k::KIND_BF16, BN, false, r9k::EPI_BF16, NP, 1, false>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
}

int na_setup(int dev) {
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (g_na[dev].ready.load(std::memory_order_acquire)) return R9K_NOALLOC_OK;
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, r9k_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    fprintf(stderr, "r9k_gemm_bf16_noalloc: scratch address lookup failed on device %d: %s\n", dev,
            cudaGetErrorString(e));
    return R9K_NOALLOC_ESETUP;
  }
  e = na_set_attr<16, 5>();
  if (e == cudaSuccess) e = na_set_attr<32, 5>();
  if (e == cudaSuccess) e = na_set_attr<64, 4>();
  if (e != cudaSuccess) {
    fprintf(stderr, "r9k_gemm_bf16_noalloc: kernel attribute set-up failed: %s\n", cudaGetErrorString(e));
    return R9K_NOALLOC_ESETUP;
  }
  if (g_na_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || fn == nullptr) {
      fprintf(stderr, "r9k_gemm_bf16_noalloc: cuTensorMapEncodeTiled unavailable\n");
      return R9K_NOALLOC_ESETUP;
    }
    g_na_encode = reinterpret_cast<r9k::EncodeTiledFn>(fn);
  }
  g_na[dev].scratch = static_cast<float*>(p);
  g_na[dev].ready.store(true, std::memory_order_release);
  return R9K_NOALLOC_OK;
}

bool na_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t K, int64_t ld, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return g_na_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int NP>
int na_launch(const CUtensorMap& ta, const CUtensorMap& tb, r9k::GemmArgs a, int S, int grid_x, float* scratch,
              cudaStream_t stream) {
  using C = r9k::GemmCfg<r9k::KIND_BF16, BN, false, NP, 1, false>;
  int* cnt = nullptr;
  float* part = nullptr;
  if (S > 1) {
    const int64_t tiles = grid_x;  // M <= 64 is one token tile
    const int64_t need = tiles * S * C::TILE_F;
    if (tiles > kNaCounterInts || need > kNaPartFloats) {
      fprintf(stderr,
              "r9k_gemm_bf16_noalloc: N=%d needs %lld bytes of split-K scratch, more than the fixed %u-byte "
              "array holds\n",
              a.N, (long long)(need * 4 + kNaCounterInts * 4), (unsigned)R9K_NOALLOC_SCRATCH_BYTES);
      return R9K_NOALLOC_ETOOLARGE;
    }
    cnt = reinterpret_cast<int*>(scratch);
    part = scratch + kNaCounterInts;
  }
  a.splits = S;
  a.kc_per_split = (a.kchunks + S - 1) / S;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid_x, S, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  // Plain stream order (no programmatic dependent launch): the kernel issues its first weight-tile
  // loads before it waits on the preceding grid, which is only safe when nothing earlier on the
  // stream is still writing w; a C caller gives no such guarantee.
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, r9k::gemm_tc_kernel<r9k::KIND_BF16, BN, false, r9k::EPI_BF16, NP, 1, false>,
                                           ta, ta, tb, a, part, cnt);
  if (e != cudaSuccess) {
    fprintf(stderr, "r9k_gemm_bf16_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return R9K_NOALLOC_ELAUNCH;
  }
  return R9K_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int r9k_gemm_bf16_noalloc(
    const void* w, int64_t ldw, const void* x, int64_t ldx, void* out, int64_t ldo, int N, int M, int K, float alpha,
    int* status, cudaStream_t stream) {
  auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (w == nullptr || x == nullptr || out == nullptr || N < 1 || M < 1 || K < 64 || K % 64 != 0 || ldw < K ||
      ldx < K || ldo < N || ldw % 8 != 0 || ldx % 8 != 0 || ldo % 8 != 0 || !aligned16(w) || !aligned16(x) ||
      !aligned16(out)) {
    fprintf(stderr, "r9k_gemm_bf16_noalloc: invalid arguments (N=%d M=%d K=%d ldw=%lld ldx=%lld ldo=%lld)\n", N, M,
            K, (long long)ldw, (long long)ldx, (long long)ldo);
    return R9K_NOALLOC_EINVAL;
  }
  if (M > 64) {
    fprintf(stderr, "r9k_gemm_bf16_noalloc: M=%d tokens; this entry point serves M <= 64\n", M);
    return R9K_NOALLOC_ETOOLARGE;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNaMaxDev) return R9K_NOALLOC_ESETUP;
  if (!g_na[dev].ready.load(std::memory_order_acquire)) {
    const int rc = na_setup(dev);
    if (rc != R9K_NOALLOC_OK) return rc;
  }
  const r9k::LaunchPlan p = r9k::plan_gemm(N, M, K / 64, false, false);
  CUtensorMap ta, tb;
  if (!na_tmap(&ta, w, N, K, ldw, 128) || !na_tmap(&tb, x, M, K, ldx, p.BN)) {
    fprintf(stderr, "r9k_gemm_bf16_noalloc: tensor-map encoding rejected the operands\n");
    return R9K_NOALLOC_EINVAL;
  }
  r9k::GemmArgs a = {};
  a.N = N; a.M = M; a.K = K; a.kchunks = K / 64;
  a.out = out; a.ldo = (int)ldo;
  a.alpha = alpha;
  a.status = status;
  a.timeout_ns = 1000000000ull;
  const int grid_x = (N + 127) / 128;
  switch (p.BN) {
    case 16: return na_launch<16, 5>(ta, tb, a, p.S, grid_x, g_na[dev].scratch, stream);
    case 32: return na_launch<32, 5>(ta, tb, a, p.S, grid_x, g_na[dev].scratch, stream);
    default: return na_launch<64, 4>(ta, tb, a, p.S, grid_x, g_na[dev].scratch, stream);
  }
}
