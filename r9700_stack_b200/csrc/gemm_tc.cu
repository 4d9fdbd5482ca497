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
// Split-K: for skinny decode GEMMs the grid's y dimension holds S splits of K grouped into one
// thread-block cluster; each CTA parks its fp32 partial tile in shared memory and the cluster's
// rank-0 CTA sums them over DSMEM in a fixed order (deterministic), then runs the epilogue.
//
// Epilogues: bf16 store (+ residual add, alpha), fp32 store, and the fused SwiGLU -> MXFP8 quant
// used by gate_up projections (two accumulators, gate and up, per CTA) that writes the down
// projection's input directly. Reference counterparts: kernels/r9k_moe_mxfp4a8.hip:187-480
// (FUSE=1 gate+up+silu), kernels/r9k_gemm_fp8.hip:36-222, kernels/r9k_moe_mxfp4a8.hip:811.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <mutex>
#include <unordered_map>
#include "common.cuh"
#include "tmap.h"

namespace r9k {

enum { KIND_BF16 = 0, KIND_MX = 1 };
enum { EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU_MXFP8 = 2 };

struct GemmArgs {
  int N;               // weight rows (output features)
  int M;               // tokens
  int K;               // reduction length (elements)
  int kchunks;         // K / chunk elements (chunk = 128 bytes of a smem row)
  int kc_per_split;    // chunks handled by one split
  uint32_t a_fmt;      // kFmtE2M1 / kFmtE4M3 for KIND_MX
  const uint8_t* sfa;  // weight scales, 512-byte chunk layout
  const uint8_t* sfa2; // second weight (dual) scales
  const uint8_t* sfb;  // activation scales
  int sf_kblocks;      // K / 32
  void* out;
  int ldo;
  const __nv_bfloat16* residual;
  int ldr;
  uint8_t* out_sf;     // SwiGLU-quant output scales
  int out_kblocks;     // (output features) / 32
  float alpha;
  int* status;
  uint64_t timeout_ns;
};

template <int KIND, int BN, bool DUAL, int STAGES>
struct GemmCfg {
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int NA = DUAL ? 2 : 1;
  static constexpr int NB_SF = (BN + 127) / 128;
  static constexpr int SFA_BYTES = (KIND == KIND_MX) ? 512 : 0;
  static constexpr int SFB_BYTES = (KIND == KIND_MX) ? 512 * NB_SF : 0;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * NA * A_BYTES;
  static constexpr int OFF_SFA = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_SFB = OFF_SFA + STAGES * NA * SFA_BYTES;
  static constexpr int OFF_BAR = (OFF_SFB + STAGES * SFB_BYTES + 15) / 16 * 16;
  static constexpr int NUM_BARS = 2 * STAGES + 1;
  static constexpr int OFF_TMEMPTR = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEMPTR + 16 + 1024;  // + alignment slack
  // TMEM columns: accumulators, then scale factors
  static constexpr int ACC_COLS = BN * NA;
  static constexpr int SFA_COL = ACC_COLS;
  static constexpr int SFB_COL = SFA_COL + 4 * NA;
  static constexpr int USED_COLS = (KIND == KIND_MX) ? SFB_COL + 4 * NB_SF : ACC_COLS;
  static constexpr int TMEM_COLS = USED_COLS <= 32 ? 32 : USED_COLS <= 64 ? 64 : USED_COLS <= 128 ? 128
                                   : USED_COLS <= 256 ? 256 : 512;
  static constexpr int PART_BYTES = 128 * BN * 4 * NA;  // split-K partial tile (fp32)
  static_assert(PART_BYTES <= OFF_SFA || BN > 64, "split-K partial must fit in the stage buffers");
};

template <int BN, bool DUAL, int EPI>
R9K_DEVINL void epilogue_chunk(const GemmArgs& a, const float* g, const float* u, int row, int tok0, int lane) {
  if constexpr (EPI == EPI_SWIGLU_MXFP8) {
    uint8_t* outq = reinterpret_cast<uint8_t*>(a.out);
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const int tok = tok0 + t;
      float h = (row < a.N) ? silu_f(g[t]) * u[t] : 0.f;
      float am = fabsf(h);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
      const int e = mx_exponent(am, 448.f);
      const uint8_t qv = f32_to_e4m3(h * exp2i(-e));
      if (tok < a.M) {
        if (row < a.N) outq[(int64_t)tok * a.ldo + row] = qv;
        if (lane == 0) a.out_sf[sf_offset(tok, row >> 5, a.out_kblocks)] = (uint8_t)(e + 127);
      }
    }
  } else if constexpr (EPI == EPI_F32) {
    float* out = reinterpret_cast<float*>(a.out);
    if (row < a.N) {
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int tok = tok0 + t;
        if (tok < a.M) out[(int64_t)tok * a.ldo + row] = g[t] * a.alpha;
      }
    }
  } else {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    if (row < a.N) {
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int tok = tok0 + t;
        if (tok < a.M) {
          float y = g[t] * a.alpha;
          if (a.residual != nullptr) y += __bfloat162float(a.residual[(int64_t)tok * a.ldr + row]);
          out[(int64_t)tok * a.ldo + row] = __float2bfloat16(y);
        }
      }
    }
  }
}

template <int KIND, int BN, bool DUAL, int EPI, int STAGES>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using C = GemmCfg<KIND, BN, DUAL, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tmem_full = empty_bar + STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEMPTR);
  __shared__ int s_abort;

  const int warp = warp_id(), lane = lane_id();
  const int m0 = blockIdx.x * 128;
  // cluster along y groups the S splits of one token tile
  const int S = (int)cluster_nctarank();
  const int split = (int)(blockIdx.y % S);
  const int n_tile = (int)(blockIdx.y / S);
  const int n0 = n_tile * BN;
  const int kc0 = split * args.kc_per_split;
  const int kc1 = min(args.kchunks, kc0 + args.kc_per_split);
  const int nk = max(0, kc1 - kc0);

  if (threadIdx.x == 0) {
    s_abort = 0;
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
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;

  constexpr uint32_t A_TX = (KIND == KIND_BF16) ? 128 * 128 : 0;  // per A tile, set below for MX
  const uint32_t a_tx = (KIND == KIND_BF16) ? A_TX : (args.a_fmt == kFmtE2M1 ? 128 * 64 : 128 * 128);
  const uint32_t stage_tx = a_tx * C::NA + BN * 128 + (KIND == KIND_MX ? 512 * C::NA + 512 * C::NB_SF : 0);
  const int box_x = (KIND == KIND_BF16) ? 64 : 128;  // elements per 128-byte smem row

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)((i / STAGES) & 1);
        if (!mbar_wait(&empty_bar[s], ph ^ 1u, args.timeout_ns)) {
          report_error(args.status, kErrMbarTimeout, 100, i);
          s_abort = 1;
          break;
        }
        const int kc = kc0 + i;
        uint8_t* sa = smem + C::OFF_A + s * C::NA * C::A_BYTES;
        uint8_t* sb = smem + C::OFF_B + s * C::B_BYTES;
        mbar_arrive_expect_tx(&full_bar[s], stage_tx);
        tma_load_2d_hint(sa, &tmA, &full_bar[s], kc * box_x, m0, pol_w);
        if (DUAL) tma_load_2d_hint(sa + C::A_BYTES, &tmA2, &full_bar[s], kc * box_x, m0, pol_w);
        tma_load_2d_hint(sb, &tmB, &full_bar[s], kc * box_x, n0, pol_x);
        if constexpr (KIND == KIND_MX) {
          uint8_t* ssfa = smem + C::OFF_SFA + s * C::NA * 512;
          uint8_t* ssfb = smem + C::OFF_SFB + s * C::SFB_BYTES;
          const int kchunks_sf = (args.sf_kblocks + 3) / 4;
          bulk_load(ssfa, args.sfa + ((int64_t)(m0 >> 7) * kchunks_sf + kc) * 512, 512, &full_bar[s]);
          if (DUAL) bulk_load(ssfa + 512, args.sfa2 + ((int64_t)(m0 >> 7) * kchunks_sf + kc) * 512, 512, &full_bar[s]);
#pragma unroll
          for (int c = 0; c < C::NB_SF; ++c)
            bulk_load(ssfb + 512 * c, args.sfb + ((int64_t)((n0 >> 7) + c) * kchunks_sf + kc) * 512, 512,
                      &full_bar[s]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)((i / STAGES) & 1);
        if (!mbar_wait(&full_bar[s], ph, args.timeout_ns)) {
          report_error(args.status, kErrMbarTimeout, 101, i);
          s_abort = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + C::OFF_A + s * C::NA * C::A_BYTES);
        const uint32_t sb = smem_u32(smem + C::OFF_B + s * C::B_BYTES);
        if constexpr (KIND == KIND_MX) {
          const uint32_t ssfa = smem_u32(smem + C::OFF_SFA + s * C::NA * 512);
          const uint32_t ssfb = smem_u32(smem + C::OFF_SFB + s * C::SFB_BYTES);
          tc_cp_32x128b_warpx4(tbase + C::SFA_COL, sdesc_sf(ssfa));
          if (DUAL) tc_cp_32x128b_warpx4(tbase + C::SFA_COL + 4, sdesc_sf(ssfa + 512));
#pragma unroll
          for (int c = 0; c < C::NB_SF; ++c) tc_cp_32x128b_warpx4(tbase + C::SFB_COL + 4 * c, sdesc_sf(ssfb + 512 * c));
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t bd = sdesc_k_sw128(sb + 32 * k);
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          if constexpr (KIND == KIND_MX) {
            const uint32_t idesc = idesc_block_scaled(args.a_fmt, kFmtE4M3, 128, BN, (uint32_t)k, (uint32_t)k);
            const uint32_t sfb_addr = (tbase + C::SFB_COL) | ((uint32_t)k << 30);
            mma_mxf8f6f4_ss(tbase, sdesc_k_sw128(sa + 32 * k), bd, idesc, acc,
                            (tbase + C::SFA_COL) | ((uint32_t)k << 30), sfb_addr);
            if (DUAL)
              mma_mxf8f6f4_ss(tbase + BN, sdesc_k_sw128(sa + C::A_BYTES + 32 * k), bd, idesc, acc,
                              (tbase + C::SFA_COL + 4) | ((uint32_t)k << 30), sfb_addr);
          } else {
            constexpr uint32_t idesc = idesc_dense(kFmtBF16, kFmtBF16, 128, BN);
            mma_f16_ss(tbase, sdesc_k_sw128(sa + 32 * k), bd, idesc, acc);
            if (DUAL) mma_f16_ss(tbase + BN, sdesc_k_sw128(sa + C::A_BYTES + 32 * k), bd, idesc, acc);
          }
        }
        tc_commit(&empty_bar[s]);
      }
      (void)ok;
      tc_commit(tmem_full);  // arrives once every MMA issued above has completed
    }
    __syncwarp();
  }

  // ------------------------------ epilogue ------------------------------
  const bool epi_warp = warp >= 2;
  const int q = warp & 3;  // TMEM lane quadrant this warp may access
  const int row_local = q * 32 + lane;
  const int row = m0 + row_local;
  float* part = reinterpret_cast<float*>(smem);  // reuses the stage buffers once the MMAs are done
  bool have_acc = false;
  if (epi_warp) {
    have_acc = mbar_wait(tmem_full, 0, args.timeout_ns);
    if (!have_acc) report_error(args.status, kErrMbarTimeout, 102, 0);
    tc_fence_after();
  }
  if (S == 1) {
    if (epi_warp && have_acc && nk > 0 && !s_abort) {
      const uint32_t trow = tbase + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float g[16], u[16];
        tmem_ld16(trow + c, g);
        if (DUAL) tmem_ld16(trow + BN + c, u);
        tmem_ld_wait();
        epilogue_chunk<BN, DUAL, EPI>(args, g, u, row, n0 + c, lane);
      }
    }
  } else {
    if (epi_warp) {
      const uint32_t trow = tbase + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float g[16], u[16];
        if (have_acc && nk > 0) {
          tmem_ld16(trow + c, g);
          if (DUAL) tmem_ld16(trow + BN + c, u);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int t = 0; t < 16; ++t) g[t] = u[t] = 0.f;
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          part[(c + t) * 128 + row_local] = g[t];
          if (DUAL) part[BN * 128 + (c + t) * 128 + row_local] = u[t];
        }
      }
    }
    cluster_sync();
    if (split == 0 && epi_warp) {
      const uint32_t base = smem_u32(part);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float g[16], u[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) g[t] = u[t] = 0.f;
        for (int r = 0; r < S; ++r) {
          const uint32_t pb = mapa_shared(base, (uint32_t)r);
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            float v;
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(pb + (uint32_t)(((c + t) * 128 + row_local) * 4)) : "memory");
            g[t] += v;
            if (DUAL) {
              asm volatile("ld.shared::cluster.f32 %0, [%1];"
                           : "=f"(v)
                           : "r"(pb + (uint32_t)((BN * 128 + (c + t) * 128 + row_local) * 4))
                           : "memory");
              u[t] += v;
            }
          }
        }
        epilogue_chunk<BN, DUAL, EPI>(args, g, u, row, n0 + c, lane);
      }
    }
    cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
struct LaunchPlan {
  int BN;
  int S;  // splits (cluster size)
  int n_tiles;
};

static int g_num_sms = 0;
static int num_sms() {
  if (g_num_sms == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return g_num_sms;
}

static LaunchPlan plan_gemm(int N, int M, int kchunks, bool dual) {
  LaunchPlan p;
  if (M <= 16) p.BN = 16;
  else if (M <= 32) p.BN = 32;
  else if (M <= 64) p.BN = 64;
  else if (M <= 128) p.BN = 128;
  else p.BN = dual ? 128 : 256;  // two accumulators of 256 columns would not fit in TMEM
  if (p.BN == 256 && M > 256) {
    // use 128-token tiles when 256-token tiles would leave SMs idle
    const int rt = (N + 127) / 128;
    if ((long)rt * ((M + 255) / 256) < num_sms()) p.BN = 128;
  }
  p.n_tiles = (M + p.BN - 1) / p.BN;
  const int row_tiles = (N + 127) / 128;
  const int tiles = row_tiles * p.n_tiles;
  p.S = 1;
  if (p.BN <= 64) {
    // split K across a cluster until about two CTAs per SM are busy; keep >= 4 chunks per split
    const int target = 2 * num_sms();
    while (p.S < 8 && tiles * p.S * 2 <= target && kchunks / (p.S * 2) >= 4) p.S *= 2;
  }
  return p;
}

template <int KIND, int BN, bool DUAL, int EPI, int STAGES>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, GemmArgs args,
                        const LaunchPlan& p, cudaStream_t stream) {
  using C = GemmCfg<KIND, BN, DUAL, STAGES>;
  auto kern = gemm_tc_kernel<KIND, BN, DUAL, EPI, STAGES>;
  static bool attr_set = false;
  if (!attr_set) {
    TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) == cudaSuccess,
                "r9k gemm: cannot set smem size");
    cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    attr_set = true;
  }
  args.kc_per_split = (args.kchunks + p.S - 1) / p.S;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((args.N + 127) / 128, p.n_tiles * p.S, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = p.S;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, ta2, tb, args);
  TORCH_CHECK(e == cudaSuccess, "r9k gemm launch failed: ", cudaGetErrorString(e));
}

template <int KIND, bool DUAL, int EPI>
static void dispatch_bn(const CUtensorMap& ta, const CUtensorMap& ta2, const CUtensorMap& tb, GemmArgs args,
                        const LaunchPlan& p, cudaStream_t st) {
  // stage counts sized for ~2 CTAs/SM on skinny tiles and 1 CTA/SM on wide tiles
  switch (p.BN) {
    case 16: launch_gemm<KIND, 16, DUAL, EPI, DUAL ? 3 : 5>(ta, ta2, tb, args, p, st); break;
    case 32: launch_gemm<KIND, 32, DUAL, EPI, DUAL ? 3 : 5>(ta, ta2, tb, args, p, st); break;
    case 64: launch_gemm<KIND, 64, DUAL, EPI, DUAL ? 2 : 4>(ta, ta2, tb, args, p, st); break;
    case 128: launch_gemm<KIND, 128, DUAL, EPI, DUAL ? 3 : 4>(ta, ta2, tb, args, p, st); break;
    default:
      if constexpr (!DUAL) launch_gemm<KIND, 256, false, EPI, 4>(ta, ta2, tb, args, p, st);
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
void gemm_mx(torch::Tensor w, torch::Tensor w_sf, bool w_fp4, torch::Tensor x, torch::Tensor x_sf,
             torch::Tensor out, c10::optional<torch::Tensor> residual, double alpha, torch::Tensor status) {
  const int64_t N = w.size(0), M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0, "gemm_mx: K must be a multiple of 128");
  TORCH_CHECK(w.size(1) == (w_fp4 ? K / 2 : K), "gemm_mx: weight/activation K mismatch");
  check_sf(w_sf, N, K, "gemm_mx weight");
  check_sf(x_sf, M, K, "gemm_mx activation");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "gemm_mx: bad out");
  const bool f32 = out.dtype() == torch::kFloat32;
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  LaunchPlan p = plan_gemm((int)N, (int)M, (int)(K / 128), false);
  check_act_sf(x_sf, p, K, "gemm_mx");
  CUtensorMap ta = w_fp4 ? tmap_fp4_kmajor(w.data_ptr(), N, K, 128) : tmap_u8_kmajor(w.data_ptr(), N, K, 128);
  CUtensorMap tb = tmap_u8_kmajor(x.data_ptr(), M, K, p.BN);
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 128);
  a.a_fmt = w_fp4 ? kFmtE2M1 : kFmtE4M3;
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
  if (f32) dispatch_bn<KIND_MX, false, EPI_F32>(ta, ta, tb, a, p, st);
  else dispatch_bn<KIND_MX, false, EPI_BF16>(ta, ta, tb, a, p, st);
}

// Fused gate/up projection + SwiGLU + MXFP8 quantisation of the result.
void gemm_mx_swiglu(torch::Tensor wg, torch::Tensor wg_sf, torch::Tensor wu, torch::Tensor wu_sf, bool w_fp4,
                    torch::Tensor x, torch::Tensor x_sf, torch::Tensor out_q, torch::Tensor out_sf,
                    torch::Tensor status) {
  const int64_t N = wg.size(0), M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0 && N % 32 == 0, "gemm_mx_swiglu: K % 128 and N % 32 required");
  TORCH_CHECK(wu.size(0) == N, "gemm_mx_swiglu: gate/up mismatch");
  check_sf(wg_sf, N, K, "swiglu gate");
  check_sf(wu_sf, N, K, "swiglu up");
  check_sf(x_sf, M, K, "swiglu act");
  check_sf(out_sf, M, N, "swiglu out");
  TORCH_CHECK(out_q.size(0) == M && out_q.size(1) == N, "gemm_mx_swiglu: bad out");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  LaunchPlan p = plan_gemm((int)N, (int)M, (int)(K / 128), true);
  check_act_sf(x_sf, p, K, "gemm_mx_swiglu");
  CUtensorMap ta = w_fp4 ? tmap_fp4_kmajor(wg.data_ptr(), N, K, 128) : tmap_u8_kmajor(wg.data_ptr(), N, K, 128);
  CUtensorMap ta2 = w_fp4 ? tmap_fp4_kmajor(wu.data_ptr(), N, K, 128) : tmap_u8_kmajor(wu.data_ptr(), N, K, 128);
  CUtensorMap tb = tmap_u8_kmajor(x.data_ptr(), M, K, p.BN);
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 128);
  a.a_fmt = w_fp4 ? kFmtE2M1 : kFmtE4M3;
  a.sfa = wg_sf.data_ptr<uint8_t>(); a.sfa2 = wu_sf.data_ptr<uint8_t>(); a.sfb = x_sf.data_ptr<uint8_t>();
  a.sf_kblocks = (int)(K / 32);
  a.out = out_q.data_ptr(); a.ldo = (int)out_q.stride(0);
  a.out_sf = out_sf.data_ptr<uint8_t>(); a.out_kblocks = (int)(N / 32);
  a.alpha = 1.f;
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
  dispatch_bn<KIND_MX, true, EPI_SWIGLU_MXFP8>(ta, ta2, tb, a, p, at::cuda::getCurrentCUDAStream());
}

// bf16 x bf16 -> bf16/f32 (kind::f16)
void gemm_bf16(torch::Tensor w, torch::Tensor x, torch::Tensor out, c10::optional<torch::Tensor> residual,
               double alpha, torch::Tensor status) {
  const int64_t N = w.size(0), M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 64 == 0 && w.size(1) == K, "gemm_bf16: K must match and be a multiple of 64");
  TORCH_CHECK(w.dtype() == torch::kBFloat16 && x.dtype() == torch::kBFloat16, "gemm_bf16: bf16 inputs");
  TORCH_CHECK(w.stride(1) == 1 && x.stride(1) == 1, "gemm_bf16: inner stride 1");
  const bool f32 = out.dtype() == torch::kFloat32;
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  LaunchPlan p = plan_gemm((int)N, (int)M, (int)(K / 64), false);
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
  if (f32) dispatch_bn<KIND_BF16, false, EPI_F32>(ta, ta, tb, a, p, st);
  else dispatch_bn<KIND_BF16, false, EPI_BF16>(ta, ta, tb, a, p, st);
}

}  // namespace r9k
