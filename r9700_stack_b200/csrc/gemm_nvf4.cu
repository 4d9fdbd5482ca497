// NVFP4 GEMM that serves the checkpoint's bits unconverted: e2m1 weights with an e4m3 scale per 16
// elements (and one fp32 global scale per tensor) times bf16 activations, on tcgen05 kind::f16.
//
//   Y[tok, row] = alpha * sum_k (e2m1[row, k] * s16[row, k / 16]) * X[tok, k]      (alpha = 1 / global)
//
// Every product e2m1 x e4m3 is exact in bf16 (at most 5 significant bits), so expanding a weight tile
// to bf16 in shared memory loses nothing, and the activations stay bf16 (no fp8 rounding of the
// input). The MXFP4 conversion the other GEMM uses re-quantises the weights instead (the reference
// measured ~1.55x the weight error for it: r9700_vllm/quant/nvfp4.py:1-22); this kernel is the
// R9K_NVFP4=native path. Reference counterpart: r9k_moe_nvfp4a8 (kernels/r9k_moe_mxfp4a8.hip:621-660).
//
// Weights are re-laid out once at load into 128-row x 64-element units, each unit one contiguous
// 4 KiB block of packed e2m1 (row r at byte 32 r) plus one 512-byte block of its scales (row r at
// byte 4 r), so a pipeline stage is two plain bulk copies. Warp roles (192 threads): warp 0 loads
// (bulk copies of the weight unit and its scales, TMA of the activation tile), warp 1 issues the
// MMAs, warps 2-5 expand each packed tile into the 128-byte-swizzled bf16 layout the MMA reads
// (thread t expands row t), then run the epilogue. Split-K: the S splits of a tile form a cluster and
// meet in distributed shared memory (S = 1, 2, 4 or 8).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "tmap.h"

namespace r9k {

enum { NVF4_EPI_BF16 = 0, NVF4_EPI_SWIGLU = 1 };

struct Nvf4Args {
  int N, M, K;           // output features, tokens, reduction
  int kchunks;           // K / 64
  int kc_per_split;
  int splits;
  const uint8_t* wq;     // [N/128][K/64][128][32] packed e2m1
  const uint8_t* ws;     // [N/128][K/64][128][4]  e4m3 scales
  const uint8_t* wq2;    // second weight (SwiGLU up) or null
  const uint8_t* ws2;
  float alpha, alpha2;   // 1 / global scale of each weight
  __nv_bfloat16* out;
  int ldo;
  int* status;
  uint64_t timeout_ns;
};

template <int BN, bool DUAL, int NP, int NC>
struct Nvf4Cfg {
  static constexpr int NA = DUAL ? 2 : 1;
  static constexpr int AP_BYTES = 128 * 32;            // packed unit
  static constexpr int AS_BYTES = 128 * 4;             // scales of the unit
  static constexpr int AC_BYTES = 128 * 128;           // expanded bf16 tile (64 elements x 2 B per row)
  static constexpr int B_BYTES = BN * 128;             // bf16 activations, 64 elements per row
  static constexpr int OFF_AP = 0;
  static constexpr int OFF_AS = OFF_AP + NP * NA * AP_BYTES;
  static constexpr int OFF_B = (OFF_AS + NP * NA * AS_BYTES + 1023) / 1024 * 1024;
  static constexpr int OFF_C = OFF_B + NP * B_BYTES;  // 1 KiB aligned (B_BYTES is a multiple of 1 KiB... for BN >= 8)
  static constexpr int OFF_BAR = OFF_C + NC * NA * AC_BYTES;
  static constexpr int NUM_BARS = 2 * NP + 2 * NC + 1;
  static constexpr int OFF_TMEMPTR = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEMPTR + 16 + 1024;
  static constexpr int ACC_COLS = BN * NA;
  static constexpr int TMEM_COLS = ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128 : 256;
  static_assert(B_BYTES % 1024 == 0, "activation tiles of 8-row swizzle atoms");
};

R9K_DEVINL float ld_dsmem_f32_nvf4(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// two e2m1 codes (low nibble = even element) -> f16x2, by the hardware conversion
R9K_DEVINL __half2 e2m1x2_to_h2(uint32_t byte) {
  uint32_t d;
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(d) : "r"(byte));
  return *reinterpret_cast<const __half2*>(&d);
}

// Expand row r of a packed unit (32 bytes = 64 e2m1 codes, low nibble first, 4 e4m3 scales) into the
// bf16 K-major tile with the 128-byte swizzle: 16-byte chunk j of the row goes to (j ^ (r & 7)).
// e2m1 x e4m3 is exact in f16 (|v| <= 2688, 5 significant bits) and in bf16.
R9K_DEVINL void expand_nvf4_row(const uint8_t* src_q, const uint8_t* src_s, uint8_t* dst, int r) {
  const uint4 q0 = reinterpret_cast<const uint4*>(src_q + r * 32)[0];
  const uint4 q1 = reinterpret_cast<const uint4*>(src_q + r * 32)[1];
  const uint32_t sc = *reinterpret_cast<const uint32_t*>(src_s + r * 4);
  const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // 8 chunks of 8 elements (one 32-bit word of codes each)
    const __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)((sc >> (8 * (j >> 1))) & 0xff), __NV_E4M3);
    const __half sh(hr);
    const __half2 s2 = __halves2half2(sh, sh);
    const uint32_t w = words[j];
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 f = __half22float2(__hmul2(e2m1x2_to_h2((w >> (8 * h)) & 0xffu), s2));
      const __nv_bfloat162 p = __float22bfloat162_rn(f);
      op[h] = *reinterpret_cast<const uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(dst + r * 128 + ((j ^ (r & 7)) << 4)) = o;
  }
}

template <int BN, bool DUAL, int EPI, int NP, int NC>
__global__ void __launch_bounds__(192, 1)
    gemm_nvf4_kernel(const __grid_constant__ CUtensorMap tmB, const Nvf4Args args) {
  using C = Nvf4Cfg<BN, DUAL, NP, NC>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* l_full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* l_empty = l_full + NP;
  uint64_t* c_full = l_empty + NP;
  uint64_t* c_empty = c_full + NC;
  uint64_t* tmem_full = c_empty + NC;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEMPTR);
  __shared__ int s_ok;

  const int warp = warp_id(), lane = lane_id();
  const int S = args.splits;
  const int split = (int)(blockIdx.y % S);
  const int n0 = (int)(blockIdx.y / S) * BN;
  const int rt = blockIdx.x;  // row tile
  const int kc0 = split * args.kc_per_split;
  const int nk = max(0, min(args.kchunks, kc0 + args.kc_per_split) - kc0);

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
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  constexpr uint32_t stage_tx = C::NA * (C::AP_BYTES + C::AS_BYTES) + C::B_BYTES;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_x = policy_evict_last();
      auto load_a = [&](int q) {
        const int s = q % NP;
        const int64_t unit = (int64_t)rt * args.kchunks + kc0 + q;
        mbar_arrive_expect_tx(&l_full[s], stage_tx);
        bulk_load(smem + C::OFF_AP + s * C::NA * C::AP_BYTES, args.wq + unit * C::AP_BYTES, C::AP_BYTES, &l_full[s]);
        bulk_load(smem + C::OFF_AS + s * C::NA * C::AS_BYTES, args.ws + unit * C::AS_BYTES, C::AS_BYTES, &l_full[s]);
        if (DUAL) {
          bulk_load(smem + C::OFF_AP + (s * C::NA + 1) * C::AP_BYTES, args.wq2 + unit * C::AP_BYTES, C::AP_BYTES,
                    &l_full[s]);
          bulk_load(smem + C::OFF_AS + (s * C::NA + 1) * C::AS_BYTES, args.ws2 + unit * C::AS_BYTES, C::AS_BYTES,
                    &l_full[s]);
        }
      };
      // weights do not depend on the previous kernel: the first stages stream before the wait
      const int npre = min(NP, nk);
      for (int q = 0; q < npre; ++q) load_a(q);
      pdl_wait();
      for (int q = 0; q < nk; ++q) {
        if (q >= npre) {
          if (!mbar_wait(&l_empty[q % NP], (uint32_t)(((q / NP) & 1) ^ 1), args.timeout_ns)) {
            report_error(args.status, kErrMbarTimeout, 120, q);
            break;
          }
          load_a(q);
        }
        tma_load_2d_hint(smem + C::OFF_B + (q % NP) * C::B_BYTES, &tmB, &l_full[q % NP], (kc0 + q) * 64, n0, pol_x);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_dense(kFmtBF16, kFmtBF16, 128, BN);
      for (int q = 0; q < nk; ++q) {
        const int s = q % NP, sc = q % NC;
        if (!mbar_wait(&l_full[s], (uint32_t)((q / NP) & 1), args.timeout_ns) ||
            !mbar_wait(&c_full[sc], (uint32_t)((q / NC) & 1), args.timeout_ns)) {
          report_error(args.status, kErrMbarTimeout, 121, q);
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + C::OFF_C + sc * C::NA * C::AC_BYTES);
        const uint32_t sb = smem_u32(smem + C::OFF_B + s * C::B_BYTES);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t acc = (q > 0 || k > 0) ? 1u : 0u;
          const uint64_t bd = sdesc_k_sw128(sb + 32 * k);
          mma_f16_ss(tbase, sdesc_k_sw128(sa + 32 * k), bd, idesc, acc);
          if (DUAL) mma_f16_ss(tbase + BN, sdesc_k_sw128(sa + C::AC_BYTES + 32 * k), bd, idesc, acc);
        }
        tc_commit(&l_empty[s]);
        tc_commit(&c_empty[sc]);
      }
      tc_commit(tmem_full);
      pdl_trigger();
    }
    __syncwarp();
  } else {
    const int ct = threadIdx.x - 64;  // 0..127: row of the tile
    // ------------------------------ expansion ------------------------------
    for (int i = 0; i < nk; ++i) {
      const int s = i % NP, sc = i % NC;
      const bool w1 = mbar_wait(&l_full[s], (uint32_t)((i / NP) & 1), args.timeout_ns);
      const bool w2 = mbar_wait(&c_empty[sc], (uint32_t)(((i / NC) & 1) ^ 1), args.timeout_ns);
      if (!w1 || !w2) {
        report_error(args.status, kErrMbarTimeout, 122, i);
        break;
      }
#pragma unroll
      for (int a = 0; a < C::NA; ++a)
        expand_nvf4_row(smem + C::OFF_AP + (s * C::NA + a) * C::AP_BYTES, smem + C::OFF_AS + (s * C::NA + a) * C::AS_BYTES,
                        smem + C::OFF_C + (sc * C::NA + a) * C::AC_BYTES, ct);
      fence_proxy_async();
      mbar_arrive(&c_full[sc]);
    }
    // ------------------------------ epilogue ------------------------------
    const int q4 = warp & 3;
    const int row_local = q4 * 32 + lane;
    const int row = rt * 128 + row_local;
    const uint32_t trow = tbase + ((uint32_t)(q4 * 32) << 16);
    pdl_wait();
    const bool wok = __all_sync(0xffffffffu, nk == 0 || mbar_wait(tmem_full, 0, args.timeout_ns));
    if (threadIdx.x == 64) s_ok = 1;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!wok && lane == 0) s_ok = 0;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const bool ok = s_ok != 0;
    if (!ok) report_error(args.status, kErrMbarTimeout, 123, 0);
    tc_fence_after();
    float* mypart = reinterpret_cast<float*>(smem);  // the load ring is idle once the accumulator is complete
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float g[16], u[16];
      if (ok && nk > 0) {
        tmem_ld16(trow + c, g);
        if (DUAL) tmem_ld16(trow + BN + c, u);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int t = 0; t < 16; ++t) g[t] = u[t] = 0.f;
      }
      if (S == 1) {
        if (ok && row < args.N) {
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const int tok = n0 + c + t;
            if (tok >= args.M) continue;
            const float y = EPI == NVF4_EPI_SWIGLU ? silu_f(g[t] * args.alpha) * (u[t] * args.alpha2) : g[t] * args.alpha;
            args.out[(int64_t)tok * args.ldo + row] = __float2bfloat16(y);
          }
        }
      } else {
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          mypart[(c + t) * 128 + row_local] = g[t];
          if (DUAL) mypart[BN * 128 + (c + t) * 128 + row_local] = u[t];
        }
      }
    }
  }

  if (S > 1) {
    // splits of the tile meet in distributed shared memory; CTA j of the cluster owns tokens t == j (mod S)
    cluster_sync();
    if (warp >= 2) {
      const int row_local = (warp & 3) * 32 + lane;
      const int row = rt * 128 + row_local;
      const uint32_t me = cluster_ctarank();
      const uint32_t base = smem_u32(smem);
      for (int t = (int)me; t < BN; t += S) {
        const int tok = n0 + t;
        if (tok >= args.M) break;
        float g = 0.f, u = 0.f;
        // every split's value requested first (all in flight together), then summed in split order
        float vg[8], vu[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (k < S) {
            const uint32_t rb = mapa_shared(base, (uint32_t)k);
            vg[k] = ld_dsmem_f32_nvf4(rb + (uint32_t)((t * 128 + row_local) * 4));
            if (DUAL) vu[k] = ld_dsmem_f32_nvf4(rb + (uint32_t)((BN * 128 + t * 128 + row_local) * 4));
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (k < S) {
            g += vg[k];
            if (DUAL) u += vu[k];
          }
        }
        if (row < args.N) {
          const float y = EPI == NVF4_EPI_SWIGLU ? silu_f(g * args.alpha) * (u * args.alpha2) : g * args.alpha;
          args.out[(int64_t)tok * args.ldo + row] = __float2bfloat16(y);
        }
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
template <int BN, bool DUAL, int EPI, int NP, int NC>
static void nvf4_launch(const CUtensorMap& tb, Nvf4Args a, int grid_x, int n_tiles, cudaStream_t st) {
  using C = Nvf4Cfg<BN, DUAL, NP, NC>;
  auto kern = gemm_nvf4_kernel<BN, DUAL, EPI, NP, NC>;
  TORCH_CHECK(ensure_smem_attr((const void*)kern, C::SMEM_BYTES) == cudaSuccess, "gemm_nvf4: smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid_x, (unsigned)(n_tiles * a.splits), 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)a.splits;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.splits > 1 ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tb, a);
  TORCH_CHECK(e == cudaSuccess, "gemm_nvf4 launch: ", cudaGetErrorString(e));
}

template <bool DUAL, int EPI>
static void nvf4_dispatch(int BN, const CUtensorMap& tb, const Nvf4Args& a, int gx, int nt, cudaStream_t st) {
  switch (BN) {
    case 16: nvf4_launch<16, DUAL, EPI, DUAL ? 4 : 6, 2>(tb, a, gx, nt, st); break;
    case 32: nvf4_launch<32, DUAL, EPI, DUAL ? 4 : 6, 2>(tb, a, gx, nt, st); break;
    case 64: nvf4_launch<64, DUAL, EPI, DUAL ? 3 : 5, 2>(tb, a, gx, nt, st); break;
    default: nvf4_launch<128, DUAL, EPI, DUAL ? 3 : 4, 2>(tb, a, gx, nt, st); break;
  }
}

// out[M, N] (bf16) = alpha * x[M, K] (bf16) @ W^T with W in NVFP4 units (see the file header); with
// wq2 the gate/up pair runs with the SwiGLU epilogue: out = silu(alpha * x Wg^T) * (alpha2 * x Wu^T).
void gemm_nvf4(torch::Tensor wq, torch::Tensor ws, double alpha, c10::optional<torch::Tensor> wq2,
               c10::optional<torch::Tensor> ws2, double alpha2, torch::Tensor x, torch::Tensor out, torch::Tensor status) {
  const int64_t M = x.size(0), K = x.size(1), N = out.size(1);
  TORCH_CHECK(x.dtype() == torch::kBFloat16 && x.stride(1) == 1 && out.dtype() == torch::kBFloat16 && out.stride(1) == 1,
              "gemm_nvf4: bf16 activations and output");
  TORCH_CHECK(K % 64 == 0 && out.size(0) == M, "gemm_nvf4: K % 64");
  const int64_t units = ((N + 127) / 128) * (K / 64);  // weight rows padded to 128 (zero codes)
  TORCH_CHECK(wq.numel() == units * 4096 && ws.numel() == units * 512 && wq.is_contiguous() && ws.is_contiguous(),
              "gemm_nvf4: weight units [N/128][K/64][128][32] and scales [N/128][K/64][128][4]");
  const bool dual = wq2.has_value() && wq2->defined();
  if (dual) TORCH_CHECK(wq2->numel() == wq.numel() && ws2->numel() == ws.numel(), "gemm_nvf4: gate / up shapes");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  const int BN = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  const int n_tiles = (int)((M + BN - 1) / BN);
  const int grid_x = (int)((N + 127) / 128);
  const int kchunks = (int)(K / 64);
  int S = 1;
  const int target = 2 * device_sm_count();
  while (S < 8 && grid_x * n_tiles * S * 2 <= target && kchunks / (S * 2) >= 4) S *= 2;
  Nvf4Args a = {};
  a.N = (int)N; a.M = (int)M; a.K = (int)K; a.kchunks = kchunks;
  a.splits = S;
  a.kc_per_split = (kchunks + S - 1) / S;
  a.wq = wq.data_ptr<uint8_t>(); a.ws = ws.data_ptr<uint8_t>();
  if (dual) { a.wq2 = wq2->data_ptr<uint8_t>(); a.ws2 = ws2->data_ptr<uint8_t>(); }
  a.alpha = (float)alpha; a.alpha2 = (float)alpha2;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = (int)out.stride(0);
  a.status = status.data_ptr<int>();
  a.timeout_ns = 1000000000ull;
  const CUtensorMap tb = tmap_bf16_kmajor(x.data_ptr(), M, K, x.stride(0), BN);
  auto st = at::cuda::getCurrentCUDAStream();
  if (dual) nvf4_dispatch<true, NVF4_EPI_SWIGLU>(BN, tb, a, grid_x, n_tiles, st);
  else nvf4_dispatch<false, NVF4_EPI_BF16>(BN, tb, a, grid_x, n_tiles, st);
}

}  // namespace r9k
