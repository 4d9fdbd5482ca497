// Mixture-of-experts kernels: routing, expert-sorted layout, activation gather and the weighted
// combine (with the gated shared expert fused in).
//
//  * moe_route: one warp per token. Mode 0 = softmax over the router logits, top-k (ties to the lower
//    expert id), optional renormalisation (Qwen / Flash-Next class; reference
//    kernels/r9k_moe_route.hip:4-31). Mode 1 = sigmoid scores plus a correction bias, group-limited
//    top-k (groups ranked by the sum of their two best biased scores), weights = unbiased scores,
//    optionally renormalised, times a routing scale (GLM / DeepSeek class; reference
//    r9700_vllm/dsv4_glue.py:180 route, kernels/r9k_dsv4_glue.hip:300 sqrt-softplus variant = mode 2).
//  * moe_align: one CTA. Counts the assignments of the local experts [e0, e0 + E_local), lays every
//    expert's rows out in a segment starting on a 128-row boundary (so MX scale chunks of the
//    activation rows line up with GEMM tiles), and emits the (expert, first row, rows) work list of
//    BN-row tiles the grouped GEMMs run over. Non-local assignments get row -1 (expert parallelism:
//    another rank owns them and the all-reduce that follows sums the partials).
//  * moe_gather: copies each assignment's MXFP8 token row (+ scale bytes) to its sorted row.
//  * moe_combine: out[t] = sum_j w[t,j] * y[row(t,j)] (+ sigmoid(shared gate) * shared[t]), fp32, one
//    rounding (reference kernels/r9k_moe_sum.hip:4-12).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

constexpr int MOE_MAX_E = 1024;
constexpr int MOE_MAX_K = 16;

// warp argmax over (value, id) pairs, ties -> lower id
R9K_DEVINL void warp_argmax(float& v, int& id) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, id, o);
    if (ov > v || (ov == v && oi < id)) { v = ov; id = oi; }
  }
}

__global__ void moe_route_kernel(const float* __restrict__ logits, int64_t ld, int T, int E, int k, int mode,
                                 const float* __restrict__ bias, int n_group, int topk_group, float scale,
                                 int renorm, int32_t* __restrict__ ids, float* __restrict__ w) {
  pdl_wait();
  extern __shared__ float sh[];  // per warp: E scores + E biased scores
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int t = blockIdx.x * (blockDim.x >> 5) + wib;
  if (t >= T) return;
  float* sc = sh + wib * 2 * E;
  float* bs = sc + E;
  const float* row = logits + (int64_t)t * ld;
  if (mode == 0) {
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) m = fmaxf(m, row[e]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    for (int e = lane; e < E; e += 32) {
      const float p = __expf(row[e] - m);
      sc[e] = p;
      s += p;
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = 1.f / s;
    for (int e = lane; e < E; e += 32) { sc[e] *= inv; bs[e] = sc[e]; }
  } else {
    for (int e = lane; e < E; e += 32) {
      const float x = row[e];
      const float s = mode == 1 ? sigmoid_f(x) : sqrtf(softplus_f(x));
      sc[e] = s;
      bs[e] = s + (bias != nullptr ? bias[e] : 0.f);
    }
    __syncwarp();
    if (n_group > 1) {
      // rank groups by the sum of their two best biased scores, keep topk_group groups
      const int gs = E / n_group;
      float gscore = -INFINITY;
      if (lane < n_group) {
        float b1 = -INFINITY, b2 = -INFINITY;
        for (int e = lane * gs; e < (lane + 1) * gs; ++e) {
          const float v = bs[e];
          if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) b2 = v;
        }
        gscore = b1 + b2;
      }
      uint32_t keep = 0;
      for (int i = 0; i < topk_group; ++i) {
        float v = (lane < n_group && !((keep >> lane) & 1u)) ? gscore : -INFINITY;
        int id = lane;
        warp_argmax(v, id);
        keep |= 1u << id;
      }
      __syncwarp();
      for (int e = lane; e < E; e += 32)
        if (!((keep >> (e / gs)) & 1u)) bs[e] = -INFINITY;
    }
  }
  __syncwarp();
  // top-k by the (biased) selection score
  float sel_w[MOE_MAX_K];
  int sel_id[MOE_MAX_K];
  float wsum = 0.f;
  for (int i = 0; i < k; ++i) {
    float v = -INFINITY;
    int id = 0x7fffffff;
    for (int e = lane; e < E; e += 32)
      if (bs[e] > v || (bs[e] == v && e < id)) { v = bs[e]; id = e; }
    warp_argmax(v, id);
    if (lane == (id & 31)) bs[id] = -INFINITY;
    __syncwarp();
    sel_id[i] = id;
    sel_w[i] = sc[id];
    wsum += sc[id];
  }
  if (lane < k) {
    float wv = 0.f;
    int iv = 0;
#pragma unroll
    for (int i = 0; i < MOE_MAX_K; ++i)
      if (i == lane) { wv = sel_w[i]; iv = sel_id[i]; }
    if (renorm) wv /= wsum;
    ids[(int64_t)t * k + lane] = iv;
    w[(int64_t)t * k + lane] = wv * scale;
  }
}

void moe_route(torch::Tensor logits, int64_t k, int64_t mode, c10::optional<torch::Tensor> bias, int64_t n_group,
               int64_t topk_group, double scale, bool renorm, torch::Tensor ids, torch::Tensor w) {
  const int64_t T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E <= MOE_MAX_E && k <= MOE_MAX_K && k <= 32 && logits.dtype() == torch::kFloat32, "moe_route: shapes");
  TORCH_CHECK(n_group <= 32 && (n_group <= 1 || E % n_group == 0), "moe_route: groups");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(logits.device());
  const int wpb = 4;
  const size_t smem = (size_t)wpb * 2 * E * sizeof(float);
  TORCH_CHECK(launch_pdl(moe_route_kernel, dim3((unsigned)((T + wpb - 1) / wpb)), dim3(32 * wpb), smem,
                         at::cuda::getCurrentCUDAStream(), logits.data_ptr<float>(), logits.stride(0), (int)T, (int)E,
                         (int)k, (int)mode, (bias.has_value() && bias->defined()) ? bias->data_ptr<float>() : nullptr,
                         (int)n_group, (int)topk_group, (float)scale, renorm ? 1 : 0, ids.data_ptr<int32_t>(),
                         w.data_ptr<float>()) == cudaSuccess,
              "moe_route launch");
}

// ------------------------------------------------------------------------------------------------
// align: counts -> 128-aligned segments -> BN-row work tiles; scatter assignment rows
// ------------------------------------------------------------------------------------------------
// exclusive scan of one value per thread over a 1024-thread block (warp shuffles + one smem pass)
R9K_DEVINL int block_exclusive_scan(int v, int* wsum, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    wsum[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  total = wsum[31];
  const int before = warp > 0 ? wsum[warp - 1] : 0;
  __syncthreads();
  return before + x - v;
}

// One CTA of 1024 threads = 32 warps; warp w owns the contiguous assignment segment w (32 segments),
// so rows come out in assignment order per expert without any serial pass:
//   1. per-segment expert counts (warp-match leaders add batch counts; no atomics across warps)
//   2. per expert: exclusive scan over segments, total count
//   3. block scans over experts: 128-aligned segment starts, BN-row tile offsets; work list
//   4. each warp re-walks its segment: row = start[e] + segment base + rank within the batch
__global__ void __launch_bounds__(1024) moe_align_kernel(const int32_t* __restrict__ ids, int A, int e0, int E_local,
                                                         int BN, int32_t* __restrict__ perm_row,
                                                         int32_t* __restrict__ seg_start, int32_t* __restrict__ work,
                                                         int32_t* __restrict__ work_count, int max_work) {
  pdl_wait();
  extern __shared__ int sm[];
  int* cnt = sm;                       // [32][E_local] counts, then segment bases
  int* start = sm + 32 * E_local;      // [E_local]
  __shared__ int wsum[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 32 * E_local; i += 1024) cnt[i] = 0;
  __syncthreads();
  const int per = (A + 31) / 32;
  const int a0 = warp * per, a1 = min(A, a0 + per);
  int* mycnt = cnt + warp * E_local;
  for (int base = a0; base < a1; base += 32) {
    const int a = base + lane;
    int e = -1 - lane;  // unique sentinel for lanes past the segment / non-local experts
    if (a < a1) {
      const int ee = ids[a] - e0;
      if (ee >= 0 && ee < E_local) e = ee;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(peers) - 1) mycnt[e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // per expert: scan over segments; thread e (one pass: E_local <= 1024)
  int total = 0;
  if (tid < E_local) {
    for (int w = 0; w < 32; ++w) {
      const int c = cnt[w * E_local + tid];
      cnt[w * E_local + tid] = total;
      total += c;
    }
  }
  int all_rows, all_tiles;
  // every work item starts on a 128-row boundary of the sorted buffer: the activation scale factors
  // are stored in 128-row chunks and a tile reads the chunk its first row falls in. With BN < 128 an
  // expert's rows are therefore spread as BN rows per 128-row slot.
  const int ntile = (total + BN - 1) / BN;
  const int padded = BN >= 128 ? (total + 127) / 128 * 128 : ntile * 128;
  const int stride = BN >= 128 ? BN : 128;
  const int st = block_exclusive_scan(tid < E_local ? padded : 0, wsum, all_rows);
  const int tl = block_exclusive_scan(tid < E_local ? ntile : 0, wsum, all_tiles);
  if (tid < E_local) {
    start[tid] = st;
    seg_start[tid] = st;
    for (int i = 0; i < ntile; ++i) {
      const int wi = tl + i;
      if (wi < max_work) {
        work[wi * 3 + 0] = tid;
        work[wi * 3 + 1] = st + i * stride;
        work[wi * 3 + 2] = min(BN, total - i * BN);
      }
    }
  }
  if (tid == 0) *work_count = min(all_tiles, max_work);
  __syncthreads();
  for (int base = a0; base < a1; base += 32) {
    const int a = base + lane;
    int e = -1 - lane;
    if (a < a1) {
      const int ee = ids[a] - e0;
      if (ee >= 0 && ee < E_local) e = ee;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (a < a1) {
      if (e >= 0) {
        const int r = mycnt[e] + __popc(peers & ((1u << lane) - 1u));  // rank within the expert
        perm_row[a] = start[e] + (BN >= 128 ? r : (r / BN) * 128 + r % BN);
      }
      else perm_row[a] = -1;
    }
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) mycnt[e] += __popc(peers);
    __syncwarp();
  }
}

void moe_align(torch::Tensor ids, int64_t e0, int64_t E_local, int64_t BN, torch::Tensor perm_row,
               torch::Tensor seg_start, torch::Tensor work, torch::Tensor work_count) {
  TORCH_CHECK(E_local <= MOE_MAX_E, "moe_align: too many local experts");
  TORCH_CHECK(BN == 16 || BN == 32 || BN == 64 || BN == 128 || BN == 256, "moe_align: BN");
  const at::cuda::CUDAGuard guard(ids.device());
  const size_t smem = (size_t)(33 * E_local) * sizeof(int);
  TORCH_CHECK(ensure_smem_attr((const void*)moe_align_kernel, 33 * MOE_MAX_E * 4) == cudaSuccess,
              "moe_align: smem attribute");
  TORCH_CHECK(launch_pdl(moe_align_kernel, dim3(1), dim3(1024), smem, at::cuda::getCurrentCUDAStream(),
                         ids.data_ptr<int32_t>(), (int)ids.numel(), (int)e0, (int)E_local, (int)BN,
                         perm_row.data_ptr<int32_t>(), seg_start.data_ptr<int32_t>(), work.data_ptr<int32_t>(),
                         work_count.data_ptr<int32_t>(), (int)work.size(0)) == cudaSuccess,
              "moe_align launch");
}

// ------------------------------------------------------------------------------------------------
// gather: sorted activation row p <- token row t (MXFP8 bytes + ue8m0 scales)
// ------------------------------------------------------------------------------------------------
__global__ void moe_gather_kernel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sf, int K, int k,
                                  const int32_t* __restrict__ perm_row, uint8_t* __restrict__ oq,
                                  uint8_t* __restrict__ osf) {
  pdl_wait();
  const int a = blockIdx.x;
  const int p = perm_row[a];
  if (p < 0) return;
  const int t = a / k;
  const int kblocks = K / 32;
  const uint4* src = reinterpret_cast<const uint4*>(q + (int64_t)t * K);
  uint4* dst = reinterpret_cast<uint4*>(oq + (int64_t)p * K);
  for (int i = threadIdx.x; i < K / 16; i += blockDim.x) dst[i] = src[i];
  for (int b = threadIdx.x; b < kblocks; b += blockDim.x) osf[sf_offset(p, b, kblocks)] = sf[sf_offset(t, b, kblocks)];
}

void moe_gather(torch::Tensor q, torch::Tensor sf, int64_t k, torch::Tensor perm_row, torch::Tensor oq,
                torch::Tensor osf) {
  const int64_t A = perm_row.numel(), K = q.size(1);
  TORCH_CHECK(K % 32 == 0, "moe_gather: K % 32");
  if (A == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(launch_pdl(moe_gather_kernel, dim3((unsigned)A), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
                         q.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>(), (int)K, (int)k, perm_row.data_ptr<int32_t>(),
                         oq.data_ptr<uint8_t>(), osf.data_ptr<uint8_t>()) == cudaSuccess,
              "moe_gather launch");
}

// ------------------------------------------------------------------------------------------------
// combine
// ------------------------------------------------------------------------------------------------
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ perm_row,
                                   const float* __restrict__ w, int k, int H, const __nv_bfloat16* __restrict__ shared,
                                   const float* __restrict__ shared_gate, __nv_bfloat16* __restrict__ out,
                                   int64_t ldo) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  float gs = 1.f;
  if (shared_gate != nullptr) gs = sigmoid_f(shared_gate[t]);
  for (int h = threadIdx.x * 2; h < H; h += blockDim.x * 2) {
    float a0 = 0.f, a1 = 0.f;
    for (int j = 0; j < k; ++j) {
      const int p = perm_row[(int64_t)t * k + j];
      if (p < 0) continue;
      const float wj = w[(int64_t)t * k + j];
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(y + (int64_t)p * H + h);
      a0 += wj * __bfloat162float(v.x);
      a1 += wj * __bfloat162float(v.y);
    }
    if (shared != nullptr) {
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(shared + (int64_t)t * H + h);
      a0 += gs * __bfloat162float(v.x);
      a1 += gs * __bfloat162float(v.y);
    }
    *reinterpret_cast<__nv_bfloat162*>(out + (int64_t)t * ldo + h) = __floats2bfloat162_rn(a0, a1);
  }
}

void moe_combine(torch::Tensor y, torch::Tensor perm_row, torch::Tensor w, int64_t k,
                 c10::optional<torch::Tensor> shared, c10::optional<torch::Tensor> shared_gate, torch::Tensor out) {
  const int64_t T = out.size(0), H = out.size(1);
  TORCH_CHECK(H % 2 == 0, "moe_combine: H even");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(launch_pdl(moe_combine_kernel, dim3((unsigned)T), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
                         reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), perm_row.data_ptr<int32_t>(),
                         w.data_ptr<float>(), (int)k, (int)H,
                         (shared.has_value() && shared->defined()) ? reinterpret_cast<const __nv_bfloat16*>(shared->data_ptr()) : nullptr,
                         (shared_gate.has_value() && shared_gate->defined()) ? shared_gate->data_ptr<float>() : nullptr,
                         reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0)) == cudaSuccess,
              "moe_combine launch");
}


// ------------------------------------------------------------------------------------------------
// bf16 gather: sorted row perm_row[a] <- token row a / k (for experts that take bf16 rows, e.g. the
// trellis-coded experts' GEMV)
// ------------------------------------------------------------------------------------------------
__global__ void moe_gather_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int H, int k,
                                       const int32_t* __restrict__ perm_row, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int a = blockIdx.x;
  const int p = perm_row[a];
  if (p < 0) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)(a / k) * ldx);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)p * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

void moe_gather_bf16(torch::Tensor x, int64_t k, torch::Tensor perm_row, torch::Tensor out) {
  const int64_t A = perm_row.numel(), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && x.stride(1) == 1 && x.stride(0) % 8 == 0 && out.is_contiguous(), "moe_gather_bf16: layout");
  if (A == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(launch_pdl(moe_gather_bf16_kernel, dim3((unsigned)A), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
                         reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), (int)H, (int)k,
                         perm_row.data_ptr<int32_t>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr())) == cudaSuccess,
              "moe_gather_bf16 launch");
}

// ------------------------------------------------------------------------------------------------
// n-gram hash ids of every token (Engram / n-gram embeddings): id_n(t) = hash(tokens t-n+1 .. t) mod
// rows for n = 2 .. 1 + n_orders. Tokens before the step's chunk come from a per-state-slot history
// of the last (max order - 1) tokens, which the kernel also advances when write_state is set
// (one thread per sequence, after the hashes of that sequence are formed).
// ------------------------------------------------------------------------------------------------
constexpr int NG_HIST = 3;

R9K_DEVINL int64_t ng_hash(const int32_t* win, int n, int order) {
  int64_t h = 0x9E3779B1LL * 0 + order;
  for (int j = 0; j < n; ++j) h = (h * 1000003LL + (int64_t)win[j] + 1) & 0x7FFFFFFFFFFFLL;
  return h;
}

__global__ void ngram_ids_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ seq_start,
                                 const int32_t* __restrict__ seq_len, const int32_t* __restrict__ seq_slot,
                                 const int32_t* __restrict__ seq_has_state, int32_t* __restrict__ hist, int S,
                                 int n_orders, int64_t rows, int write_state, int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= S) return;
  const int t0 = seq_start[s], n = seq_len[s], slot = seq_slot[s];
  int32_t win[NG_HIST + 1];
  const bool hs = seq_has_state[s] != 0;
  for (int j = 0; j < NG_HIST; ++j) win[j] = hs ? hist[slot * NG_HIST + j] : -1;  // oldest first
  for (int i = 0; i < n; ++i) {
    for (int j = 0; j < NG_HIST - 1; ++j) win[j] = win[j + 1];
    win[NG_HIST - 1] = ids[t0 + i];
    // order o uses the last o tokens of the window (missing history hashes as -1)
    for (int o = 0; o < n_orders; ++o) {
      const int order = o + 2;
      int32_t w[NG_HIST];
      for (int j = 0; j < order; ++j) w[j] = win[NG_HIST - order + j];
      out[(int64_t)(t0 + i) * n_orders + o] = ng_hash(w, order, order) % rows;
    }
  }
  if (write_state)
    for (int j = 0; j < NG_HIST; ++j) hist[slot * NG_HIST + j] = win[j];
}

void ngram_ids(torch::Tensor ids, torch::Tensor seq_start, torch::Tensor seq_len, torch::Tensor seq_slot,
               torch::Tensor seq_has_state, torch::Tensor hist, int64_t n_orders, int64_t rows, bool write_state,
               torch::Tensor out) {
  const int64_t S = seq_start.size(0);
  if (S == 0) return;
  TORCH_CHECK(n_orders >= 1 && n_orders + 1 <= NG_HIST, "ngram_ids: orders 2..3");
  TORCH_CHECK(hist.size(1) == NG_HIST && out.dtype() == torch::kInt64, "ngram_ids: hist [slots, 3], out int64");
  const at::cuda::CUDAGuard guard(ids.device());
  TORCH_CHECK(launch_pdl(ngram_ids_kernel, dim3((unsigned)((S + 63) / 64)), dim3(64), 0, at::cuda::getCurrentCUDAStream(),
                         ids.data_ptr<int32_t>(), seq_start.data_ptr<int32_t>(), seq_len.data_ptr<int32_t>(),
                         seq_slot.data_ptr<int32_t>(), seq_has_state.data_ptr<int32_t>(), hist.data_ptr<int32_t>(),
                         (int)S, (int)n_orders, rows, write_state ? 1 : 0, out.data_ptr<int64_t>()) == cudaSuccess,
              "ngram_ids launch");
}

}  // namespace r9k
