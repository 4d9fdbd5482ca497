// QSA sparse attention for the full-attention layers of the Flash-Next class (Qwen4Exp): every query
// row attends to the indexer's top-k complete 4-token groups plus the causal tail of the group it sits
// in, instead of its whole context.
//
// Per attention layer two small caches sit beside the paged fp8 K/V (same block table, 64 rows a page):
//   ktok [blocks][64][128] bf16  every token's indexer key (after its norm and rope)
//   ckey [blocks][64][128] e4m3  group g's compressed key = mean of its 4 token keys, stored at row g
//                                (a sequence's groups use the first quarter of its pages)
// Per query row t at position p (ctx = p + 1):
//   vis      = ctx / 4 complete groups
//   score[g] = sum_h relu(q_idx[t, h] . ckey[g]) / sqrt(128)       g < vis   (indexer_score kernel)
//   sel      = the top-k groups by score, in group order (all of them when vis <= k)  (topk_select)
//   keys     = the 4 tokens of every selected group, then tokens [4 * vis, p] (the open group's tail)
//   out      = softmax(q . K_keys * scale) V_keys, per query head, times sigmoid(gate)
// Kernels: qsa_key_write (token keys into ktok), qsa_compress (rows that close a group write its
// compressed key), qsa_attn (rows x kv heads x splits over the gathered key list, CUDA cores, online
// softmax in fp32) and qsa_combine (LSE merge of the splits, output gate, bf16 store).
// When every row's vis <= k the selection is the whole causal context: the model then runs its
// dense attention kernels instead and skips scoring entirely.
// (reference: kernels/r9k_qsa.hip:11-30 semantics -- group bitmap + causal tail, split + LSE merge;
// kernels/r9k_qsa_score.hip:9-27 -- indexer score over the visible compressed columns.)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

constexpr int QSA_D = 256;    // attention head dim
constexpr int QSA_ID = 128;   // indexer dim
constexpr int QSA_KT = 32;    // keys per tile
constexpr int QSA_GMAX = 16;  // query heads per kv head

// one warp per row: 128 bf16 = 16 lanes x 16 bytes
__global__ void qsa_key_write_kernel(const __nv_bfloat16* __restrict__ ik, int64_t ld, const int32_t* __restrict__ slots,
                                     __nv_bfloat16* __restrict__ ktok, int T) {
  pdl_wait();
  pdl_trigger();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= T || lane >= 16) return;
  const int slot = slots[w];
  if (slot < 0) return;
  reinterpret_cast<uint4*>(ktok + (int64_t)slot * QSA_ID)[lane] =
      reinterpret_cast<const uint4*>(ik + (int64_t)w * ld)[lane];
}

// one warp per row; rows whose context ends on a group boundary write that group's compressed key
__global__ void qsa_compress_kernel(const __nv_bfloat16* __restrict__ ktok, const int32_t* __restrict__ bt, int mb,
                                    const int32_t* __restrict__ tok_seq, const int32_t* __restrict__ tok_ctx,
                                    uint8_t* __restrict__ ckey, int T) {
  pdl_wait();
  pdl_trigger();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= T) return;
  const int ctx = tok_ctx[w], seq = tok_seq[w];
  if (ctx <= 0 || seq < 0 || (ctx & 3)) return;
  const int g = ctx / 4 - 1;
  const int32_t* row = bt + (int64_t)seq * mb;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int tok = 4 * g + j;
    const __nv_bfloat16* src = ktok + ((int64_t)row[tok >> 6] * 64 + (tok & 63)) * QSA_ID + 4 * lane;
    const uint2 v = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += __bfloat162float(h[i]);
  }
  uint8_t* dst = ckey + ((int64_t)row[g >> 6] * 64 + (g & 63)) * QSA_ID + 4 * lane;
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) packed |= (uint32_t)f32_to_e4m3(acc[i] * 0.25f) << (8 * i);
  *reinterpret_cast<uint32_t*>(dst) = packed;
}

struct QsaArgs {
  const __nv_bfloat16* q;
  int64_t ldq;  // row stride of q (elements); heads are contiguous 256-element rows
  const uint8_t* kc;
  const uint8_t* vc;
  const int32_t* bt;
  int mb;
  const int32_t* tok_seq;
  const int32_t* tok_ctx;
  const int32_t* sel;
  int64_t ld_sel;
  const int32_t* count;
  int hq, hkv, G, nsplit;
  float scale;  // sm_scale * k_scale * log2(e)
  float* part_o;  // nsplit > 1: unnormalised partials and (max, sum) per (row, head, split)
  float* part_ml;
  __nv_bfloat16* out;  // nsplit == 1: the kernel writes the gated bf16 output itself
  int64_t ldo;
  const __nv_bfloat16* gate;
  int64_t ldg;
  float v_scale;
};

// grid (T, hkv, nsplit), 256 threads, GP = query heads per kv head padded to 8 or 16. Per 32-key tile:
//   gather   fp8 K and V rows into shared memory (16 bytes per thread per pass)
//   scores   warp w owns keys 4w .. 4w + 3: each lane decodes 8 dims of the key once and dots them
//            with every head's query; a butterfly reduction leaves head h's sum in lanes of that head
//   softmax  warp w owns heads w (and w + 8): online max / sum over the tile, p -> p_t[key][head]
//   P V      warp w owns dims 32w .. 32w + 31 for every head: each V element is decoded once
// so every fp8 element is converted once per tile, not once per head.
template <int GP>
__global__ void __launch_bounds__(256) qsa_attn_kernel(const QsaArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ __align__(16) float q_s[GP][QSA_D];
  // K and V tiles, double-buffered (tile i + 1 loads during tile i): 32 KB of dynamic shared memory
  extern __shared__ __align__(16) uint8_t qsa_dyn[];
  auto k_s = reinterpret_cast<uint8_t(*)[QSA_KT][QSA_D]>(qsa_dyn);
  auto v_s = reinterpret_cast<uint8_t(*)[QSA_KT][QSA_D]>(qsa_dyn + 2 * QSA_KT * QSA_D);
  __shared__ __align__(16) float s_s[GP][QSA_KT];  // scores of the tile, by head
  __shared__ __align__(16) float p_t[QSA_KT][GP];  // probabilities, by key
  __shared__ float corr_s[GP], m_s[GP], l_s[GP];
  const int t = blockIdx.x, h = blockIdx.y, sp = blockIdx.z, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.G;
  const int seq = a.tok_seq[t], ctx = a.tok_ctx[t];
  const int vis = ctx / 4, cnt = min(a.count[t], vis);
  const int L = 4 * cnt + (ctx - 4 * vis);
  const int ntile = (L + QSA_KT - 1) / QSA_KT;
  const int tps = (ntile + a.nsplit - 1) / a.nsplit;
  const int t0 = sp * tps, t1 = min(ntile, t0 + tps);
  const int32_t* row = a.bt + (int64_t)seq * a.mb;
  const int32_t* sel = a.sel + (int64_t)t * a.ld_sel;
  for (int i = tid; i < GP * QSA_D; i += 256) {
    const int hh = i / QSA_D, d = i - hh * QSA_D;
    q_s[hh][d] = hh < G ? __bfloat162float(a.q[(int64_t)t * a.ldq + (int64_t)(h * G + hh) * QSA_D + d]) : 0.f;
  }
  // head-warp state (heads warp, warp + 8) and dim-warp accumulators (dim 32 warp + lane, every head)
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[GP];
#pragma unroll
  for (int j = 0; j < GP; ++j) o[j] = 0.f;
  const int dim = 32 * warp + lane;
  // gather of one tile into buffer b: 16 bytes of K and of V per thread per pass, zero-filled past the
  // key list (every thread derives its key's token itself, so no extra barrier is needed)
  auto issue = [&](int tile, int b) {
    const int j0 = tile * QSA_KT, nk = min(QSA_KT, L - j0);
    for (int i = tid; i < QSA_KT * 16; i += 256) {
      const int kk = i >> 4, c = i & 15;
      const int j = j0 + kk;
      int64_t off = 0;
      uint32_t bytes = 0;
      if (kk < nk) {
        const int tok = j < 4 * cnt ? 4 * sel[j >> 2] + (j & 3) : 4 * vis + (j - 4 * cnt);
        off = (((int64_t)row[tok >> 6] * a.hkv + h) * 64 + (tok & 63)) * QSA_D + 16 * c;
        bytes = 16;
      }
      const uint32_t dk = static_cast<uint32_t>(__cvta_generic_to_shared(&k_s[b][kk][16 * c]));
      const uint32_t dv = static_cast<uint32_t>(__cvta_generic_to_shared(&v_s[b][kk][16 * c]));
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dk), "l"(a.kc + off), "r"(bytes) : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dv), "l"(a.vc + off), "r"(bytes) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (t0 < t1) issue(t0, 0);
  for (int tile = t0; tile < t1; ++tile) {
    const int j0 = tile * QSA_KT, nk = min(QSA_KT, L - j0);
    const int b = (tile - t0) & 1;
    __syncthreads();  // the previous tile's shared reads are done (buffer b ^ 1 is free)
    if (tile + 1 < t1) issue(tile + 1, b ^ 1);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    // scores: 4 keys per warp, lane = 8 dims
#pragma unroll 1
    for (int kq = 0; kq < 4; ++kq) {
      const int kk = 4 * warp + kq;
      const uint2 raw = *reinterpret_cast<const uint2*>(&k_s[b][kk][8 * lane]);
      float kf[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kf[i] = e4m3_to_f32((uint8_t)(raw.x >> (8 * i)));
        kf[4 + i] = e4m3_to_f32((uint8_t)(raw.y >> (8 * i)));
      }
      float v[GP];
#pragma unroll
      for (int hh = 0; hh < GP; ++hh) {
        const float4 qa = *reinterpret_cast<const float4*>(&q_s[hh][8 * lane]);
        const float4 qb = *reinterpret_cast<const float4*>(&q_s[hh][8 * lane + 4]);
        v[hh] = qa.x * kf[0] + qa.y * kf[1] + qa.z * kf[2] + qa.w * kf[3] + qb.x * kf[4] + qb.y * kf[5] +
                qb.z * kf[6] + qb.w * kf[7];
      }
      // butterfly: each step halves the values a lane holds (lanes with the mask bit keep the upper half)
#pragma unroll
      for (int n = GP, m = 16; n > 1; n >>= 1, m >>= 1) {
        const bool up = lane & m;
#pragma unroll
        for (int j = 0; j < n / 2; ++j) {
          const float keep = up ? v[j + n / 2] : v[j];
          const float send = up ? v[j] : v[j + n / 2];
          v[j] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
      }
      // lanes sharing the remaining low bits hold the same head's partials: finish the sum over them
      constexpr int LOWB = GP == 16 ? 2 : 4;  // lanes per head after the butterfly
#pragma unroll
      for (int m = LOWB / 2; m >= 1; m >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
      // step with mask m kept the upper half in lanes with bit m set, so the head is lane / LOWB
      const int head = lane / LOWB;
      if ((lane & (LOWB - 1)) == 0) s_s[head][kk] = v[0];
    }
    __syncthreads();
    // softmax: head-warps, lane = key
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int hh = warp + 8 * j;
      if (hh >= GP) break;
      const float sc = (lane < nk && hh < G) ? s_s[hh][lane] * a.scale : -INFINITY;
      float mx = sc;
#pragma unroll
      for (int k = 16; k; k >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, k));
      const float mn = fmaxf(m_run[j], mx);
      const float pv = (mn == -INFINITY) ? 0.f : exp2f(sc - mn);
      float ps = pv;
#pragma unroll
      for (int k = 16; k; k >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, k);
      const float corr = (mn == -INFINITY) ? 1.f : exp2f(m_run[j] - mn);
      l_run[j] = l_run[j] * corr + ps;
      m_run[j] = mn;
      p_t[lane][hh] = pv;
      if (lane == 0) corr_s[hh] = corr;
    }
    __syncthreads();
    // P V: dim-warps, lane = dim
#pragma unroll
    for (int hh = 0; hh < GP; ++hh) o[hh] *= corr_s[hh];
    for (int kk = 0; kk < nk; ++kk) {
      const float vf = e4m3_to_f32(v_s[b][kk][dim]);
#pragma unroll
      for (int hq4 = 0; hq4 < GP / 4; ++hq4) {
        const float4 pp = *reinterpret_cast<const float4*>(&p_t[kk][4 * hq4]);
        o[4 * hq4 + 0] += pp.x * vf;
        o[4 * hq4 + 1] += pp.y * vf;
        o[4 * hq4 + 2] += pp.z * vf;
        o[4 * hq4 + 3] += pp.w * vf;
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  // hand the head-warps' (max, sum) to the dim-warps
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int hh = warp + 8 * j;
    if (hh < GP && lane == 0) {
      m_s[hh] = m_run[j];
      l_s[hh] = l_run[j];
    }
  }
  __syncthreads();
  if (a.nsplit == 1) {
#pragma unroll
    for (int hh = 0; hh < GP; ++hh) {
      if (hh >= G) break;
      const int qh = h * G + hh;
      float y = l_s[hh] > 0.f ? o[hh] * (a.v_scale / l_s[hh]) : 0.f;
      if (a.gate != nullptr) {
        const float g = __bfloat162float(a.gate[(int64_t)t * a.ldg + (int64_t)qh * QSA_D + dim]);
        y *= 1.f / (1.f + __expf(-g));
      }
      a.out[(int64_t)t * a.ldo + (int64_t)qh * QSA_D + dim] = __float2bfloat16(y);
    }
    return;
  }
#pragma unroll
  for (int hh = 0; hh < GP; ++hh) {
    if (hh >= G) break;
    const int64_t r = (int64_t)t * a.hq + h * G + hh;
    a.part_o[(r * a.nsplit + sp) * QSA_D + dim] = o[hh];
    if (tid == 0) {
      a.part_ml[(r * a.nsplit + sp) * 2 + 0] = m_s[hh];
      a.part_ml[(r * a.nsplit + sp) * 2 + 1] = l_s[hh];
    }
  }
}

// one CTA of 256 threads per (row, query head): LSE merge over the splits, v scale, output gate
__global__ void __launch_bounds__(256) qsa_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                                          int nsplit, int hq, float v_scale,
                                                          const __nv_bfloat16* __restrict__ gate, int64_t ldg,
                                                          __nv_bfloat16* __restrict__ out, int64_t ldo) {
  pdl_wait();
  pdl_trigger();
  const int64_t r = blockIdx.x;
  const int t = (int)(r / hq), hh = (int)(r % hq), d = threadIdx.x;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, part_ml[(r * nsplit + s) * 2]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float ms = part_ml[(r * nsplit + s) * 2];
    if (ms == -INFINITY) continue;
    const float w = exp2f(ms - mx);
    den += w * part_ml[(r * nsplit + s) * 2 + 1];
    num += w * part_o[(r * nsplit + s) * QSA_D + d];
  }
  float y = den > 0.f ? num / den * v_scale : 0.f;
  if (gate != nullptr) {
    const float g = __bfloat162float(gate[(int64_t)t * ldg + (int64_t)hh * QSA_D + d]);
    y *= 1.f / (1.f + __expf(-g));
  }
  out[(int64_t)t * ldo + (int64_t)hh * QSA_D + d] = __float2bfloat16(y);
}

void qsa_key_write(torch::Tensor ik, torch::Tensor slots, torch::Tensor ktok) {
  const int64_t T = ik.size(0);
  if (T == 0) return;
  TORCH_CHECK(ik.size(1) == QSA_ID && ik.stride(1) == 1 && ik.stride(0) % 8 == 0 && ik.dtype() == torch::kBFloat16,
              "qsa_key_write: ik [T, 128] bf16, 16-byte aligned rows");
  TORCH_CHECK(ktok.size(-1) == QSA_ID && ktok.dtype() == torch::kBFloat16 && ktok.is_contiguous(), "qsa_key_write: ktok");
  const at::cuda::CUDAGuard guard(ik.device());
  launch_pdl(qsa_key_write_kernel, dim3((unsigned)((T * 32 + 255) / 256)), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(ik.data_ptr()), ik.stride(0), slots.data_ptr<int32_t>(),
             reinterpret_cast<__nv_bfloat16*>(ktok.data_ptr()), (int)T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qsa_compress(torch::Tensor ktok, torch::Tensor block_table, torch::Tensor tok_seq, torch::Tensor tok_ctx,
                  torch::Tensor ckey) {
  const int64_t T = tok_ctx.size(0);
  if (T == 0) return;
  TORCH_CHECK(ckey.dtype() == torch::kUInt8 && ckey.size(-1) == QSA_ID && ckey.is_contiguous(), "qsa_compress: ckey");
  const at::cuda::CUDAGuard guard(ktok.device());
  launch_pdl(qsa_compress_kernel, dim3((unsigned)((T * 32 + 255) / 256)), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(ktok.data_ptr()), block_table.data_ptr<int32_t>(),
             (int)block_table.size(1), tok_seq.data_ptr<int32_t>(), tok_ctx.data_ptr<int32_t>(),
             ckey.data_ptr<uint8_t>(), (int)T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qsa_attention(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_table,
                   torch::Tensor tok_seq, torch::Tensor tok_ctx, torch::Tensor sel, torch::Tensor count,
                   double sm_scale, double k_scale, double v_scale, int64_t nsplit, torch::Tensor part_o,
                   torch::Tensor part_ml, c10::optional<torch::Tensor> gate, torch::Tensor out) {
  const int64_t T = q.size(0), hq = q.size(1);
  if (T == 0) return;
  const int64_t hkv = kc.size(1);
  TORCH_CHECK(q.size(2) == QSA_D && q.stride(2) == 1 && q.stride(1) == QSA_D && q.dtype() == torch::kBFloat16,
              "qsa_attention: q [T, hq, 256] bf16");
  TORCH_CHECK(kc.dim() == 4 && kc.size(2) == 64 && kc.size(3) == QSA_D && kc.is_contiguous() && vc.is_contiguous() &&
                  kc.sizes() == vc.sizes() && kc.dtype() == torch::kUInt8,
              "qsa_attention: fp8 caches [blocks, hkv, 64, 256]");
  TORCH_CHECK(hq % hkv == 0 && hq / hkv <= QSA_GMAX, "qsa_attention: at most 16 query heads per kv head");
  TORCH_CHECK(nsplit == 1 || (nsplit > 1 && part_o.numel() >= T * hq * nsplit * QSA_D &&
                                 part_ml.numel() >= T * hq * nsplit * 2 && part_o.is_contiguous() && part_ml.is_contiguous()),
              "qsa_attention: split partials");
  TORCH_CHECK(sel.dtype() == torch::kInt32 && sel.stride(1) == 1 && count.dtype() == torch::kInt32, "qsa_attention: sel");
  TORCH_CHECK(out.size(0) == T && out.size(1) == hq * QSA_D && out.stride(1) == 1 && out.dtype() == torch::kBFloat16,
              "qsa_attention: out [T, hq * 256] bf16");
  QsaArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.ldq = q.stride(0);
  a.kc = kc.data_ptr<uint8_t>();
  a.vc = vc.data_ptr<uint8_t>();
  a.bt = block_table.data_ptr<int32_t>();
  a.mb = (int)block_table.size(1);
  a.tok_seq = tok_seq.data_ptr<int32_t>();
  a.tok_ctx = tok_ctx.data_ptr<int32_t>();
  a.sel = sel.data_ptr<int32_t>();
  a.ld_sel = sel.stride(0);
  a.count = count.data_ptr<int32_t>();
  a.hq = (int)hq;
  a.hkv = (int)hkv;
  a.G = (int)(hq / hkv);
  a.nsplit = (int)nsplit;
  a.scale = (float)(sm_scale * k_scale * 1.4426950408889634);
  a.part_o = part_o.data_ptr<float>();
  a.part_ml = part_ml.data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  const __nv_bfloat16* g = nullptr;
  int64_t ldg = 0;
  if (gate.has_value() && gate->defined()) {
    TORCH_CHECK(gate->stride(1) == 1 && gate->size(1) == hq * QSA_D && gate->stride(0) % 8 == 0,
                "qsa_attention: gate [T, hq * 256], 16-byte aligned rows");
    g = reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr());
    ldg = gate->stride(0);
  }
  TORCH_CHECK(out.stride(0) % 8 == 0, "qsa_attention: out rows 16-byte aligned");
  a.gate = g;
  a.ldg = ldg;
  a.v_scale = (float)v_scale;
  const at::cuda::CUDAGuard guard(q.device());
  auto st = at::cuda::getCurrentCUDAStream();
  constexpr int dyn = 4 * QSA_KT * QSA_D;
  TORCH_CHECK(ensure_smem_attr((const void*)qsa_attn_kernel<8>, dyn) == cudaSuccess &&
                  ensure_smem_attr((const void*)qsa_attn_kernel<16>, dyn) == cudaSuccess,
              "qsa_attention: shared memory attribute");
  if (a.G <= 8) launch_pdl(qsa_attn_kernel<8>, dim3((unsigned)T, (unsigned)hkv, (unsigned)nsplit), dim3(256), dyn, st, a);
  else launch_pdl(qsa_attn_kernel<16>, dim3((unsigned)T, (unsigned)hkv, (unsigned)nsplit), dim3(256), dyn, st, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (nsplit == 1) return;
  launch_pdl(qsa_combine_kernel, dim3((unsigned)(T * hq)), dim3(256), 0, st, a.part_o, a.part_ml, (int)nsplit, (int)hq,
             (float)v_scale, g, ldg, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace r9k
