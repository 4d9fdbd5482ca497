// Prefill-sized MX and bf16 GEMMs with the token dimension on the MMA's M side ("swap AB").
//
// out[M, N] = X[M, K] W[N, K]^T. The skinny-GEMM kernel (gemm_tc.cu) puts 128 weight rows on TMEM
// lanes, so its epilogue thread owns one output feature and writes it for every token: 2-byte stores
// strided by the output row, ~15 us of a ~35 us 128 x 256 tile at M = 8192 (measured with the phase
// trace). Here a CTA computes 128 tokens x BNW features with A = the activation tile (MXFP8) and B = the
// weight tile (MXFP4 or MXFP8): TMEM lane = token, so each epilogue thread holds 16 consecutive features
// per tcgen05.ld and stores them as 16-byte vectors (the residual add reads the same way).
// Warp roles as in gemm_tc.cu: warp 0 TMA producer (weights for the first stages before the
// programmatic-dependent-launch wait, activations after), warp 1 MMA issuer (tcgen05.mma
// kind::mxf8f6f4.block_scale, scale factors copied to TMEM per stage), warps 2-5 epilogue.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "gemm_common.cuh"
#include "tmap.h"

namespace r9k {

template <int KIND, int BNW, int NP>
struct SwapCfg {
  static constexpr int A_BYTES = 128 * 128;        // 128 tokens x 128 fp8
  static constexpr int B_BYTES = BNW * 128;        // BNW weight rows x 128 elements (1 byte each in smem)
  static constexpr int NB = BNW / 128;             // weight row tiles per CTA
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + NP * A_BYTES;
  static constexpr int OFF_SFA = OFF_B + NP * B_BYTES;
  static constexpr int SF_A = KIND == KIND_MX ? 512 : 0;   // scale-factor bytes per stage (MX only)
  static constexpr int OFF_SFB = OFF_SFA + NP * SF_A;
  static constexpr int OFF_BAR = OFF_SFB + NP * SF_A * NB;
  static constexpr int NUM_BARS = 2 * NP + 1;
  static constexpr int OFF_TMEMPTR = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEMPTR + 16 + 1024;
  static constexpr int SF_STRIDE = 4 + 4 * NB;    // TMEM columns of one stage's scale factors
  static constexpr int SFA_COL = BNW;
  static constexpr int SFB_COL = BNW + 4;
  static constexpr int USED = BNW + (KIND == KIND_MX ? NP * SF_STRIDE : 0);
  static constexpr int TMEM_COLS = USED <= 256 ? 256 : 512;
};

template <int KIND, int BNW, int EPI, int NP>
__global__ void __launch_bounds__(192, 1)
    gemm_swap_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, GemmArgs args) {
  using C = SwapCfg<KIND, BNW, NP>;
  constexpr bool MX = KIND == KIND_MX;
  constexpr int KBOX = MX ? 128 : 64;  // elements of K per stage (128-byte smem rows)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* l_full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* l_empty = l_full + NP;
  uint64_t* tmem_full = l_empty + NP;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEMPTR);
  __shared__ int s_ok;
  const int warp = warp_id(), lane = lane_id();
  const int f0 = blockIdx.x * BNW;  // first output feature (weight row)
  const int t0 = blockIdx.y * 128;  // first token
  const int nk = args.kchunks;
  const int kchunks_sf = (args.sf_kblocks + 3) / 4;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NP; ++i) {
      mbar_init(&l_full[i], 1);
      mbar_init(&l_empty[i], 1);
    }
    mbar_init(tmem_full, 1);
    fence_mbar_init();
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  // weight row tiles of this CTA inside N (a tile past N is neither loaded nor used: its columns are
  // masked in the epilogue, and its scale-factor chunk would lie outside the scale tensor)
  const int nb = min(C::NB, (args.N - f0 + 127) / 128);
  const uint32_t w_tx =
      (uint32_t)((MX && args.a_fmt == kFmtE2M1 ? 128 * 64 : 128 * 128) + C::SF_A) * (uint32_t)nb;
  const uint32_t stage_tx = w_tx + 128 * 128 + C::SF_A;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      auto load_w = [&](int q) {
        const int s = q % NP;
        mbar_arrive_expect_tx(&l_full[s], stage_tx);
#pragma unroll
        for (int b = 0; b < C::NB; ++b) {
          if (b >= nb) break;
          const int rows0 = f0 + b * 128;
          load_a_tile(smem + C::OFF_B + s * C::B_BYTES + b * 128 * 128, &tmW, &l_full[s], args, q, KBOX, rows0, pol_w);
          if constexpr (MX)
            bulk_load(smem + C::OFF_SFB + (s * C::NB + b) * 512,
                      args.sfa + ((int64_t)(rows0 >> 7) * kchunks_sf + q) * 512, 512, &l_full[s]);
        }
      };
      auto load_x = [&](int q) {
        const int s = q % NP;
        tma_load_2d_hint(smem + C::OFF_A + s * C::A_BYTES, &tmX, &l_full[s], q * KBOX, t0, pol_x);
        if constexpr (MX)
          bulk_load(smem + C::OFF_SFA + s * 512, args.sfb + ((int64_t)(t0 >> 7) * kchunks_sf + q) * 512, 512,
                    &l_full[s]);
      };
      const int npre = min(NP, nk);
      for (int q = 0; q < npre; ++q) load_w(q);  // weights do not depend on the previous kernel
      pdl_wait();
      for (int q = 0; q < nk; ++q) {
        if (q >= npre) {
          if (!mbar_wait(&l_empty[q % NP], (uint32_t)(((q / NP) & 1) ^ 1), args.timeout_ns)) {
            report_error(args.status, kErrMbarTimeout, 130, q);
            break;
          }
          load_w(q);
        }
        load_x(q);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      for (int q = 0; q < nk; ++q) {
        const int s = q % NP;
        if (!mbar_wait(&l_full[s], (uint32_t)((q / NP) & 1), args.timeout_ns)) {
          report_error(args.status, kErrMbarTimeout, 131, q);
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + C::OFF_A + s * C::A_BYTES);
        const uint32_t sb = smem_u32(smem + C::OFF_B + s * C::B_BYTES);
        if constexpr (MX) {
          const uint32_t sfo = (uint32_t)(s * C::SF_STRIDE);
          tc_cp_32x128b_warpx4(tbase + C::SFA_COL + sfo, sdesc_sf(smem_u32(smem + C::OFF_SFA + s * 512)));
#pragma unroll
          for (int b = 0; b < C::NB; ++b)
            tc_cp_32x128b_warpx4(tbase + C::SFB_COL + sfo + 4 * b,
                                 sdesc_sf(smem_u32(smem + C::OFF_SFB + (s * C::NB + b) * 512)));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t idesc = idesc_block_scaled(kFmtE4M3, args.a_fmt, 128, BNW, (uint32_t)k, (uint32_t)k);
            mma_mxf8f6f4_ss(tbase, sdesc_k_sw128(sa + 32 * k), sdesc_k_sw128(sb + 32 * k), idesc,
                            (q > 0 || k > 0) ? 1u : 0u, (tbase + C::SFA_COL + sfo) | ((uint32_t)k << 30),
                            (tbase + C::SFB_COL + sfo) | ((uint32_t)k << 30));
          }
        } else {
          constexpr uint32_t idesc = idesc_dense(kFmtBF16, kFmtBF16, 128, BNW);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16_ss(tbase, sdesc_k_sw128(sa + 32 * k), sdesc_k_sw128(sb + 32 * k), idesc, (q > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&l_empty[s]);
      }
      tc_commit(tmem_full);
      pdl_trigger();
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue: thread = token ------------------------------
    const int q4 = warp & 3;
    const int tok = t0 + q4 * 32 + lane;
    const uint32_t trow = tbase + ((uint32_t)(q4 * 32) << 16);
    pdl_wait();
    const bool wok = __all_sync(0xffffffffu, nk == 0 || mbar_wait(tmem_full, 0, args.timeout_ns));
    if (threadIdx.x == 64) s_ok = 1;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!wok && lane == 0) s_ok = 0;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const bool ok = s_ok != 0;
    if (!ok) report_error(args.status, kErrMbarTimeout, 132, 0);
    tc_fence_after();
#pragma unroll 1
    for (int c = 0; c < BNW; c += 16) {
      float v[16];
      if (ok && nk > 0) {
        tmem_ld16(trow + c, v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
      }
      const int f = f0 + c;
      if (tok >= args.M || f >= args.N) continue;
      if constexpr (EPI == EPI_F32) {
        float* o = reinterpret_cast<float*>(args.out) + (int64_t)tok * args.ldo + f;
        if (f + 16 <= args.N) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(o + i) =
                make_float4(v[i] * args.alpha, v[i + 1] * args.alpha, v[i + 2] * args.alpha, v[i + 3] * args.alpha);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (f + i < args.N) o[i] = v[i] * args.alpha;
        }
      } else {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(args.out) + (int64_t)tok * args.ldo + f;
        float y[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = v[i] * args.alpha;
        if (f + 16 <= args.N) {
          if (args.residual != nullptr) {
            const __nv_bfloat16* r = args.residual + (int64_t)tok * args.ldr + f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint4 rv = *reinterpret_cast<const uint4*>(r + 8 * h);
              const __nv_bfloat162* rb = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 rf = __bfloat1622float2(rb[j]);
                y[8 * h + 2 * j] += rf.x;
                y[8 * h + 2 * j + 1] += rf.y;
              }
            }
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 pk;
            uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const __nv_bfloat162 b2 = __floats2bfloat162_rn(y[8 * h + 2 * j], y[8 * h + 2 * j + 1]);
              pw[j] = *reinterpret_cast<const uint32_t*>(&b2);
            }
            *reinterpret_cast<uint4*>(o + 8 * h) = pk;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (f + i >= args.N) continue;
            float yi = y[i];
            if (args.residual != nullptr) yi += __bfloat162float(args.residual[(int64_t)tok * args.ldr + f + i]);
            o[i] = __float2bfloat16(yi);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

template <int KIND>
static bool swap_launch(const CUtensorMap& tx, const CUtensorMap& tw, GemmArgs& a, bool f32, int64_t M, int64_t N) {
  constexpr int BNW = 256, NP = 4;
  using Cfg = SwapCfg<KIND, BNW, NP>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + BNW - 1) / BNW), (unsigned)((M + 127) / 128));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (f32) {
    auto kern = gemm_swap_kernel<KIND, BNW, EPI_F32, NP>;
    TORCH_CHECK(ensure_smem_attr((const void*)kern, Cfg::SMEM_BYTES) == cudaSuccess, "gemm swap: smem");
    e = cudaLaunchKernelEx(&cfg, kern, tx, tw, a);
  } else {
    auto kern = gemm_swap_kernel<KIND, BNW, EPI_BF16, NP>;
    TORCH_CHECK(ensure_smem_attr((const void*)kern, Cfg::SMEM_BYTES) == cudaSuccess, "gemm swap: smem");
    e = cudaLaunchKernelEx(&cfg, kern, tx, tw, a);
  }
  TORCH_CHECK(e == cudaSuccess, "gemm swap launch: ", cudaGetErrorString(e));
  return true;
}

// the vector epilogue wants 16-byte aligned output / residual rows
static bool swap_fits(const torch::Tensor& out, const c10::optional<torch::Tensor>& residual) {
  const int esz = out.dtype() == torch::kFloat32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) || (out.stride(0) * esz) % 16) return false;
  if (residual.has_value() && residual->defined() &&
      ((reinterpret_cast<uintptr_t>(residual->data_ptr()) & 15) || (residual->stride(0) * 2) % 16))
    return false;
  return true;
}

static void swap_common(GemmArgs& a, torch::Tensor& out, const c10::optional<torch::Tensor>& residual, double alpha,
                        torch::Tensor& status) {
  a.out = out.data_ptr(); a.ldo = (int)out.stride(0);
  if (residual.has_value() && residual->defined()) {
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ldr = (int)residual->stride(0);
  }
  a.alpha = (float)alpha;
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
}

// x: e4m3 [M, K] + chunk scales; w: MX weight (row-major [N, K/2 | K] or tiled units) + chunk scales.
// Returns false (nothing launched) where the shapes or strides do not fit the vector epilogue.
bool gemm_mx_swap(const CUtensorMap& tw, const torch::Tensor& x, const torch::Tensor& x_sf, const torch::Tensor& w_sf,
                  bool w_fp4, bool w_tiled, torch::Tensor& out, const c10::optional<torch::Tensor>& residual, double alpha,
                  torch::Tensor& status) {
  const int64_t N = out.size(1), M = x.size(0), K = x.size(1);
  if (!swap_fits(out, residual)) return false;
  if (x_sf.numel() < ((M + 127) / 128) * ((K / 32 + 3) / 4) * 512) return false;
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 128);
  a.a_fmt = w_fp4 ? kFmtE2M1 : kFmtE4M3;
  a.a_tiled = w_tiled ? 1 : 0;
  a.sfa = w_sf.data_ptr<uint8_t>();  // weight scales (B operand here)
  a.sfb = x_sf.data_ptr<uint8_t>();  // activation scales (A operand here)
  a.sf_kblocks = (int)(K / 32);
  swap_common(a, out, residual, alpha, status);
  const CUtensorMap tx = tmap_u8_kmajor(x.data_ptr(), M, K, 128);
  return swap_launch<KIND_MX>(tx, tw, a, out.dtype() == torch::kFloat32, M, N);
}

// bf16 x [M, K] (row stride ldx) times bf16 w [N, K] (row stride ldw)
bool gemm_bf16_swap(const torch::Tensor& w, const torch::Tensor& x, torch::Tensor& out,
                    const c10::optional<torch::Tensor>& residual, double alpha, torch::Tensor& status) {
  const int64_t N = w.size(0), M = x.size(0), K = x.size(1);
  if (!swap_fits(out, residual)) return false;
  GemmArgs a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = (int)(K / 64);
  a.a_tiled = 0;
  swap_common(a, out, residual, alpha, status);
  const CUtensorMap tx = tmap_bf16_kmajor(x.data_ptr(), M, K, x.stride(0), 128);
  const CUtensorMap tw = tmap_bf16_kmajor(w.data_ptr(), N, K, w.stride(0), 128);
  return swap_launch<KIND_BF16>(tx, tw, a, out.dtype() == torch::kFloat32, M, N);
}

}  // namespace r9k
