// Persistent stream-K tcgen05 GEMM for skinny (decode) batches: M <= 64 tokens.
//
// At decode sizes a linear layer is a weight stream: the kernel is bound by how many weight bytes
// are in flight per SM. One CTA runs per SM with an 8-11 stage TMA ring (~200 KB of shared memory),
// and the weight tiles are cut into "units" of 128 rows x 128 K elements, dealt out evenly:
// CTA p takes units [p U / P, (p+1) U / P) in row-tile-major order, so every SM streams the same
// number of bytes regardless of the matrix shape (no wave quantisation, no idle SMs).
//
// A CTA's range covers whole tiles and at most two partial tiles (its first and last). Each
// partial accumulator goes to a per-CTA slot of a fp32 workspace; the last contributor to finish
// a tile (per-tile arrival counter, self-resetting) sums the contributors' slots in CTA order --
// a fixed order, so results are deterministic -- and runs the epilogue. Accumulators of a CTA's
// tiles live side by side in TMEM.
//
// Same operand formats, descriptors and epilogues as the tiled kernel (gemm_tc.cu).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "gemm_common.cuh"

namespace r9k {

struct SkArgs {
  int U;            // total units = row_tiles * kchunks
  int P;            // CTAs
  int nseg_max;     // accumulator slots per CTA
  float* part;      // [P][2][NA][BN][128] fp32
  int* counters;    // [row_tiles], zero between calls
};

R9K_DEVINL int sk_owner(int u, int P, int U) { return (int)((((int64_t)u + 1) * P + U - 1) / U) - 1; }

template <int KIND, int BN, bool DUAL, int STAGES>
struct SkCfg {
  static constexpr int NA = DUAL ? 2 : 1;
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int SFA_BYTES = (KIND == KIND_MX) ? 512 : 0;
  static constexpr int SFB_BYTES = (KIND == KIND_MX) ? 512 : 0;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * NA * A_BYTES;
  static constexpr int OFF_SFA = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_SFB = OFF_SFA + STAGES * NA * SFA_BYTES;
  static constexpr int OFF_BAR = (OFF_SFB + STAGES * SFB_BYTES + 15) / 16 * 16;
  static constexpr int OFF_TMEMPTR = OFF_BAR + (2 * STAGES + 1) * 8;
  static constexpr int SMEM_BYTES = OFF_TMEMPTR + 16 + 1024;
  static constexpr int TILE_F = NA * BN * 128;  // floats per partial tile
  static_assert(BN <= 64, "stream-K kernel serves skinny batches");
};

template <int KIND, int BN, bool DUAL, int EPI, int STAGES>
__global__ void __launch_bounds__(192, 1)
    gemm_sk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB, const GemmArgs args, const SkArgs sk) {
  using C = SkCfg<KIND, BN, DUAL, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tmem_full = empty_bar + STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEMPTR);
  __shared__ int s_last, s_ok;

  const int warp = warp_id(), lane = lane_id();
  const int p = blockIdx.x;
  const int KC = args.kchunks;
  const int u0 = (int)((int64_t)p * sk.U / sk.P);
  const int u1 = (int)((int64_t)(p + 1) * sk.U / sk.P);
  const int nk = u1 - u0;
  const int t_first = u0 / KC;
  const int nseg = nk > 0 ? (u1 - 1) / KC - t_first + 1 : 0;
  const int acc_cols = sk.nseg_max * BN * C::NA;
  const int sfa_col = acc_cols, sfb_col = acc_cols + 4 * C::NA;
  int tcols = 32;
  while (tcols < sfb_col + 4) tcols <<= 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    mbar_init(tmem_full, 1);
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (DUAL) prefetch_tmap(&tmA2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, (uint32_t)tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const uint32_t a_tx = (KIND == KIND_BF16) ? 128 * 128 : (args.a_fmt == kFmtE2M1 ? 128 * 64 : 128 * 128);
  const uint32_t stage_tx = a_tx * C::NA + BN * 128 + (KIND == KIND_MX ? 512 * C::NA + 512 : 0);
  const int box_x = (KIND == KIND_BF16) ? 64 : 128;
  const int kchunks_sf = (args.sf_kblocks + 3) / 4;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      auto load_a = [&](int i) {
        const int s = i % STAGES;
        const int u = u0 + i;
        const int t = u / KC, kc = u % KC;
        uint8_t* sa = smem + C::OFF_A + s * C::NA * C::A_BYTES;
        mbar_arrive_expect_tx(&full_bar[s], stage_tx);
        load_a_tile(sa, &tmA, &full_bar[s], args, kc, box_x, t * 128, pol_w);
        if (DUAL) load_a_tile(sa + C::A_BYTES, &tmA2, &full_bar[s], args, kc, box_x, t * 128, pol_w);
        if constexpr (KIND == KIND_MX) {
          uint8_t* ssfa = smem + C::OFF_SFA + s * C::NA * 512;
          bulk_load(ssfa, args.sfa + ((int64_t)t * kchunks_sf + kc) * 512, 512, &full_bar[s]);
          if (DUAL) bulk_load(ssfa + 512, args.sfa2 + ((int64_t)t * kchunks_sf + kc) * 512, 512, &full_bar[s]);
        }
      };
      auto load_b = [&](int i) {
        const int s = i % STAGES;
        const int kc = (u0 + i) % KC;
        tma_load_2d_hint(smem + C::OFF_B + s * C::B_BYTES, &tmB, &full_bar[s], kc * box_x, 0, pol_x);
        if constexpr (KIND == KIND_MX)
          bulk_load(smem + C::OFF_SFB + s * 512, args.sfb + (int64_t)kc * 512, 512, &full_bar[s]);
      };
      const int npre = min(STAGES, nk);
      for (int i = 0; i < npre; ++i) load_a(i);  // weights stream before the predecessor finishes
      pdl_wait();
      for (int i = 0; i < nk; ++i) {
        if (i >= npre) {
          if (!mbar_wait(&empty_bar[i % STAGES], (uint32_t)(((i / STAGES) & 1) ^ 1), args.timeout_ns)) {
            report_error(args.status, kErrMbarTimeout, 110, i);
            break;
          }
          load_a(i);
        }
        load_b(i);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&full_bar[s], (uint32_t)((i / STAGES) & 1), args.timeout_ns)) {
          report_error(args.status, kErrMbarTimeout, 111, i);
          break;
        }
        tc_fence_after();
        const int u = u0 + i;
        const int seg = u / KC - t_first;
        const bool first = (i == 0) || (u % KC == 0);
        const uint32_t dacc = tbase + (uint32_t)(seg * BN * C::NA);
        const uint32_t sa = smem_u32(smem + C::OFF_A + s * C::NA * C::A_BYTES);
        const uint32_t sb = smem_u32(smem + C::OFF_B + s * C::B_BYTES);
        if constexpr (KIND == KIND_MX) {
          const uint32_t ssfa = smem_u32(smem + C::OFF_SFA + s * C::NA * 512);
          tc_cp_32x128b_warpx4(tbase + sfa_col, sdesc_sf(ssfa));
          if (DUAL) tc_cp_32x128b_warpx4(tbase + sfa_col + 4, sdesc_sf(ssfa + 512));
          tc_cp_32x128b_warpx4(tbase + sfb_col, sdesc_sf(smem_u32(smem + C::OFF_SFB + s * 512)));
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t bd = sdesc_k_sw128(sb + 32 * k);
          const uint32_t acc = (!first || k > 0) ? 1u : 0u;
          if constexpr (KIND == KIND_MX) {
            const uint32_t idesc = idesc_block_scaled(args.a_fmt, kFmtE4M3, 128, BN, (uint32_t)k, (uint32_t)k);
            const uint32_t sfb_addr = (tbase + sfb_col) | ((uint32_t)k << 30);
            mma_mxf8f6f4_ss(dacc, sdesc_k_sw128(sa + 32 * k), bd, idesc, acc, (tbase + sfa_col) | ((uint32_t)k << 30),
                            sfb_addr);
            if (DUAL)
              mma_mxf8f6f4_ss(dacc + BN, sdesc_k_sw128(sa + C::A_BYTES + 32 * k), bd, idesc, acc,
                              (tbase + sfa_col + 4) | ((uint32_t)k << 30), sfb_addr);
          } else {
            constexpr uint32_t idesc = idesc_dense(kFmtBF16, kFmtBF16, 128, BN);
            mma_f16_ss(dacc, sdesc_k_sw128(sa + 32 * k), bd, idesc, acc);
            if (DUAL) mma_f16_ss(dacc + BN, sdesc_k_sw128(sa + C::A_BYTES + 32 * k), bd, idesc, acc);
          }
        }
        tc_commit(&empty_bar[s]);
      }
      tc_commit(tmem_full);
      pdl_trigger();
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue (warps 2..5) ------------------------------
    const int q = warp & 3;
    const int row_local = q * 32 + lane;
    const uint32_t trow = tbase + ((uint32_t)(q * 32) << 16);
    pdl_wait();
    const bool wok = __all_sync(0xffffffffu, nk == 0 || mbar_wait(tmem_full, 0, args.timeout_ns));
    // the four epilogue warps agree on one outcome, so the named barriers below stay matched
    if (threadIdx.x == 64) s_ok = 1;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!wok && lane == 0) s_ok = 0;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const bool ok = s_ok != 0;
    tc_fence_after();
    for (int seg = 0; seg < nseg && ok; ++seg) {
      const int t = t_first + seg;
      const int ka = (seg == 0) ? u0 % KC : 0;
      const int kb = (seg == nseg - 1) ? (u1 - 1) % KC + 1 : KC;
      const int row = t * 128 + row_local;
      const uint32_t tacc = trow + (uint32_t)(seg * BN * C::NA);
      if (ka == 0 && kb == KC) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float g[16], u[16];
          tmem_ld16(tacc + c, g);
          if (DUAL) tmem_ld16(tacc + BN + c, u);
          tmem_ld_wait();
          epilogue_chunk<BN, DUAL, EPI>(args, g, u, row, c, lane);
        }
        continue;
      }
      // partial tile: park it in this CTA's slot (0 = first segment, 1 = last segment)
      const int slot = (seg == 0) ? 0 : 1;
      float* mypart = sk.part + ((int64_t)p * 2 + slot) * C::TILE_F;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float g[16], u[16];
        tmem_ld16(tacc + c, g);
        if (DUAL) tmem_ld16(tacc + BN + c, u);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          mypart[(c + i) * 128 + row_local] = g[i];
          if (DUAL) mypart[BN * 128 + (c + i) * 128 + row_local] = u[i];
        }
      }
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int pf = sk_owner(t * KC, sk.P, sk.U);
      const int pl = sk_owner((t + 1) * KC - 1, sk.P, sk.U);
      if (threadIdx.x == 64) {
        const int old = atomicAdd(&sk.counters[t], 1);
        s_last = (old == pl - pf) ? 1 : 0;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (!s_last) continue;
      __threadfence();
      // last contributor: sum every contributor's slot in CTA order, then the epilogue
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float g[16], u[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) g[i] = u[i] = 0.f;
        for (int qq = pf; qq <= pl; ++qq) {
          const int qslot = ((int)((int64_t)qq * sk.U / sk.P) / KC < t) ? 1 : 0;
          const float* src = sk.part + ((int64_t)qq * 2 + qslot) * C::TILE_F;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            g[i] += __ldcg(src + (c + i) * 128 + row_local);
            if (DUAL) u[i] += __ldcg(src + BN * 128 + (c + i) * 128 + row_local);
          }
        }
        epilogue_chunk<BN, DUAL, EPI>(args, g, u, row, c, lane);
      }
      if (threadIdx.x == 64) sk.counters[t] = 0;
    }
    if (!ok) report_error(args.status, kErrMbarTimeout, 112, 0);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, (uint32_t)tcols);
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
static int sk_num_sms() { return device_sm_count(); }

static int sk_ctas_per_sm() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("R9K_SK_CPS");
    v = e ? std::max(1, std::min(4, atoi(e))) : 2;
  }
  return v;
}

template <int KIND, int BN, bool DUAL, int EPI, int STAGES>
static bool sk_launch(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, const GemmArgs& args,
                      float* part, int64_t part_floats, int* counters, int64_t ncounters, cudaStream_t st, int cps) {
  using C = SkCfg<KIND, BN, DUAL, STAGES>;
  const int row_tiles = (args.N + 127) / 128;
  const int U = row_tiles * args.kchunks;
  int P = std::min(sk_num_sms() * cps, U);
  // accumulator slots: a CTA spans at most ceil(units/KC) + 1 tiles; they must fit TMEM
  auto nseg_for = [&](int P_) { return (U / P_ + 1 + args.kchunks - 1) / args.kchunks + 1; };
  int nseg = nseg_for(P);
  if (nseg * BN * C::NA + 4 * C::NA + 4 > 512) return false;
  if ((int64_t)P * 2 * C::TILE_F > part_floats || row_tiles > ncounters) return false;
  if (STAGES < 2) return false;
  SkArgs sk{U, P, nseg, part, counters};
  auto kern = gemm_sk_kernel<KIND, BN, DUAL, EPI, STAGES>;
  TORCH_CHECK(ensure_smem_attr((const void*)kern, C::SMEM_BYTES) == cudaSuccess, "gemm_sk: smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)P, 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, ta2, tb, args, sk);
  TORCH_CHECK(e == cudaSuccess, "gemm_sk launch failed: ", cudaGetErrorString(e));
  return true;
}

// Dispatch a skinny GEMM (M <= 64) to the stream-K kernel. Returns false when the shape does not fit
// (the caller then uses the tiled kernel).
template <int KIND, bool DUAL, int EPI>
bool gemm_sk_dispatch(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, const GemmArgs& a,
                      torch::Tensor& ws, cudaStream_t st) {
  if (a.M > 64) return false;
  float* part = ws.data_ptr<float>();
  // workspace layout: [counters: 65536 ints][partials]
  int* counters = reinterpret_cast<int*>(part);
  const int64_t ncounters = 65536;
  float* parts = part + ncounters;
  const int64_t part_floats = ws.numel() - ncounters;
  // CTAs per SM (R9K_SK_CPS, default 2): each CTA runs its own TMA/MMA pipeline, and the shared memory
  // of the SM is split between them
  const int cps = sk_ctas_per_sm();
#define R9K_SK(BN_, S1, S2, S3)                                                                                     \
  switch (cps) {                                                                                                  \
    case 1: return sk_launch<KIND, BN_, DUAL, EPI, S1>(ta, ta2, tb, a, parts, part_floats, counters, ncounters, st, 1); \
    case 2: return sk_launch<KIND, BN_, DUAL, EPI, S2>(ta, ta2, tb, a, parts, part_floats, counters, ncounters, st, 2); \
    default: return sk_launch<KIND, BN_, DUAL, EPI, S3>(ta, ta2, tb, a, parts, part_floats, counters, ncounters, st, 3); \
  }
  if (a.M <= 16) { if (DUAL) { R9K_SK(16, 6, 3, 2) } else { R9K_SK(16, 11, 5, 3) } }
  if (a.M <= 32) { if (DUAL) { R9K_SK(32, 5, 2, 1) } else { R9K_SK(32, 10, 5, 3) } }
  if (DUAL) { R9K_SK(64, 5, 2, 1) } else { R9K_SK(64, 8, 4, 2) }
#undef R9K_SK
}

template bool gemm_sk_dispatch<KIND_MX, false, EPI_BF16>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                                        const GemmArgs&, torch::Tensor&, cudaStream_t);
template bool gemm_sk_dispatch<KIND_MX, false, EPI_F32>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                                       const GemmArgs&, torch::Tensor&, cudaStream_t);
template bool gemm_sk_dispatch<KIND_MX, true, EPI_SWIGLU_MXFP8>(const CUtensorMap&, const CUtensorMap&,
                                                               const CUtensorMap&, const GemmArgs&, torch::Tensor&,
                                                               cudaStream_t);
template bool gemm_sk_dispatch<KIND_BF16, false, EPI_BF16>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                                          const GemmArgs&, torch::Tensor&, cudaStream_t);
template bool gemm_sk_dispatch<KIND_BF16, false, EPI_F32>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                                         const GemmArgs&, torch::Tensor&, cudaStream_t);

}  // namespace r9k
