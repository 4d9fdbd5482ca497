// Shared definitions of the tcgen05 GEMM kernels (tiled: gemm_tc.cu, stream-K: gemm_sk.cu).
#pragma once
#include "common.cuh"
#include "comm.cuh"
#include "tmap.h"

namespace r9k {

enum { KIND_BF16 = 0, KIND_MX = 1 };
enum { EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU_MXFP8 = 2, EPI_PUSH = 3, EPI_SWIGLU_BF16 = 4 };

struct GemmArgs {
  int N;               // weight rows (output features)
  int M;               // tokens
  int K;               // reduction length (elements)
  int kchunks;         // K / chunk elements (chunk = 128 bytes of a smem row)
  int kc_per_split;    // chunks handled by one split
  int splits;          // K splits (tiled kernel)
  uint32_t a_fmt;      // kFmtE2M1 / kFmtE4M3 for KIND_MX
  int a_tiled;         // weights stored as contiguous 128x128 units (3-D tensor map)
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
  // EPI_PUSH: the bf16 result goes to slot [rank] of every rank's all-reduce region (NVLink stores)
  ArPeers peers;
  int ar_call;
  int ar_ll;  // EPI_PUSH into the LL slots (epoch in every word, no tile flags)
  // grouped (MoE) mode: grid.y walks a device work list of (expert, first row, rows) token tiles;
  // expert e's weight is row tiles [e * g_row_tiles, (e + 1) * g_row_tiles) of the stacked matrix
  const int32_t* g_work;
  const int32_t* g_count;
  int g_row_tiles;
  // weight chunks prefetched into L2 ahead of the shared-memory ring (0: none)
  int l2_prefetch;
  // split-K with the S splits of a tile launched as one thread-block cluster (1, S, 1): the fp32
  // partials meet in distributed shared memory instead of a global workspace (no fix-up kernel tail)
  int cluster_k;
  // tuning trace (null unless set with gemm_trace): per CTA, %globaltimer at kernel entry, set-up
  // done, producer past the programmatic wait, first stage landed, last MMA issued, accumulator
  // complete (epilogue), CTA done (epilogue thread; slot 7: the same seen by thread 0); cluster split-K:
  // partial parked, first cluster barrier passed, reduced + stored, second barrier passed
  unsigned long long* trace;
};
enum { kTrEntry = 0, kTrSetup, kTrPdl, kTrFirst, kTrIssued, kTrAcc, kTrDone, kTrDone0, kTrParked, kTrSync1,
       kTrReduced, kTrSync2, kTrN = 12 };

R9K_DEVINL float4 ld_dsmem_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr) : "memory");
  return v;
}

R9K_DEVINL float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// A (weight) tile load: row-major 2-D map, or pre-tiled 3-D map indexed by unit
R9K_DEVINL void load_a_tile(void* dst, const CUtensorMap* map, uint64_t* bar, const GemmArgs& a, int kc, int box_x,
                            int m0, uint64_t pol) {
  if (a.a_tiled) tma_load_3d_hint(dst, map, bar, 0, 0, (m0 >> 7) * a.kchunks + kc, pol);
  else tma_load_2d_hint(dst, map, bar, kc * box_x, m0, pol);
}

R9K_DEVINL void prefetch_a_tile(const CUtensorMap* map, const GemmArgs& a, int kc, int box_x, int m0) {
  if (a.a_tiled) tma_prefetch_3d(map, 0, 0, (m0 >> 7) * a.kchunks + kc);
  else tma_prefetch_2d(map, kc * box_x, m0);
}

// tmask: bit t set = token tok0 + t is stored by this thread's CTA (cluster split-K spreads a tile's
// tokens over the CTAs of the cluster)
template <int BN, bool DUAL, int EPI>
R9K_DEVINL void epilogue_chunk(const GemmArgs& a, const float* g, const float* u, int row, int tok0, int lane,
                               const ArCall* arc = nullptr, uint32_t tmask = 0xffffu) {
  if constexpr (EPI == EPI_SWIGLU_MXFP8) {
    uint8_t* outq = reinterpret_cast<uint8_t*>(a.out);
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const int tok = tok0 + t;
      if (!((tmask >> t) & 1u)) continue;  // uniform across the warp: the shuffles below stay converged
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
  } else if constexpr (EPI == EPI_PUSH) {
    if (row < a.N) {
      const int W = a.peers.world;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int tok = tok0 + t;
        if (tok < a.M) {
          const __nv_bfloat16 v = __float2bfloat16(g[t] * a.alpha);
          const int64_t off = (int64_t)tok * a.N + row;
#pragma unroll
          for (int p = 0; p < AR_MAX_WORLD; ++p)
            if (p < W) arc->dst[p][off] = v;
        }
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU_BF16) {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    if (row < a.N) {
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int tok = tok0 + t;
        if (tok < a.M && ((tmask >> t) & 1u)) out[(int64_t)tok * a.ldo + row] = __float2bfloat16(silu_f(g[t]) * u[t]);
      }
    }
  } else if constexpr (EPI == EPI_F32) {
    float* out = reinterpret_cast<float*>(a.out);
    if (row < a.N) {
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int tok = tok0 + t;
        if (tok < a.M && ((tmask >> t) & 1u)) out[(int64_t)tok * a.ldo + row] = g[t] * a.alpha;
      }
    }
  } else {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    if (row < a.N) {
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int tok = tok0 + t;
        if (tok < a.M && ((tmask >> t) & 1u)) {
          float y = g[t] * a.alpha;
          if (a.residual != nullptr) y += __bfloat162float(a.residual[(int64_t)tok * a.ldr + row]);
          out[(int64_t)tok * a.ldo + row] = __float2bfloat16(y);
        }
      }
    }
  }
}

}  // namespace r9k
