// Device-side LRU cache of MoE experts whose weights live in pinned host memory.
//
// Each MoE layer keeps S device slots of expert weights (gate / up / down in the grouped GEMM's tiled
// MX layout). Per step, entirely on the device (so it runs inside CUDA graphs):
//   lru_route: one CTA. Marks the experts this step routes to, refreshes the stamps of the resident
//     ones, and for the missing ones picks victims among the slots no routed expert occupies --
//     free slots first, then the least recently used, ties to the lower slot (a deterministic choice,
//     identical on every rank that sees the same routing). It rewrites the expert -> slot maps, emits
//     the miss list, counts hits and misses, and converts the routing's expert ids into slot ids.
//   expert_copy: copies each missed expert's bytes from host memory (UVA) into its slot; the grid has
//     one CTA row per possible miss, and CTAs past the miss count exit.
// A step that needs more distinct experts than there are slots records a kConfig error in the status
// word (the capacity must cover one step's experts).
// (reference: kernels/third_party/davetha/r4d_lru.hip lru_manage_k / lru_gather_k, r9700_vllm/moe/cache.py
// LayerCache -- written here from the algorithm: deterministic victim ranking and a miss list.)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

constexpr int LRU_MAX = 1024;

__global__ void __launch_bounds__(1024) lru_route_kernel(
    const int32_t* __restrict__ ids, int A, int e0, int E, int S, int32_t* __restrict__ slot_of,
    int32_t* __restrict__ expert_of, int64_t* __restrict__ stamp, int64_t* __restrict__ clock,
    int32_t* __restrict__ miss_e, int32_t* __restrict__ miss_s, int32_t* __restrict__ miss_count,
    int64_t* __restrict__ counters, int32_t* __restrict__ slot_ids, int* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  __shared__ int need[LRU_MAX];
  __shared__ int rank_of[LRU_MAX];
  __shared__ unsigned long long key[LRU_MAX];
  __shared__ int s_wsum[32];
  __shared__ int s_nmiss, s_ncand;
  __shared__ long long s_now;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_now = (long long)(clock[0] + 1);
  for (int e = tid; e < E; e += 1024) need[e] = 0;
  __syncthreads();
  for (int a = tid; a < A; a += 1024) {
    const int e = ids[a] - e0;
    if (e >= 0 && e < E) need[e] = 1;
  }
  __syncthreads();
  const long long now = s_now;
  // misses in ascending expert order: exclusive scan of (needed and not resident), one expert per thread
  const int e = tid;
  const int miss = (e < E && need[e] && slot_of[e] < 0) ? 1 : 0;
  if (e < E && need[e] && slot_of[e] >= 0) stamp[slot_of[e]] = now;
  int x = miss;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = s_wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_wsum[lane] = w;
  }
  __syncthreads();
  const int excl = (warp > 0 ? s_wsum[warp - 1] : 0) + x - miss;
  if (e < E) rank_of[e] = miss ? excl : -1;
  if (tid == 0) s_nmiss = s_wsum[31];
  // victim keys: slots holding no routed expert, ordered by (stamp, slot); free slots stamp -1
  for (int s = tid; s < LRU_MAX; s += 1024) {
    unsigned long long k = ~0ull;
    if (s < S) {
      const int ex = expert_of[s];
      if (ex < 0) k = (unsigned long long)s;  // free: before every stamped slot
      else if (!need[ex]) k = ((unsigned long long)(stamp[s] + 1) << 11) | (unsigned long long)s;
    }
    key[s] = k;
  }
  __syncthreads();
  // bitonic sort of the LRU_MAX keys (ascending)
  for (int size = 2; size <= LRU_MAX; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < LRU_MAX; i += 1024) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = key[i], b = key[j];
          if ((a > b) == up) {
            key[i] = b;
            key[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  if (tid == 0) {
    int nc = 0;
    while (nc < S && key[nc] != ~0ull) ++nc;
    s_ncand = nc;
    if (s_nmiss > nc) report_error(status, kErrConfig, 500, s_nmiss);
  }
  __syncthreads();
  const int nmiss = min(s_nmiss, s_ncand);
  if (e < E && miss && rank_of[e] < nmiss) {
    const int v = (int)(key[rank_of[e]] & 2047ull);
    const int old = expert_of[v];
    if (old >= 0) slot_of[old] = -1;
  }
  __syncthreads();
  if (e < E && miss && rank_of[e] < nmiss) {
    const int r = rank_of[e];
    const int v = (int)(key[r] & 2047ull);
    expert_of[v] = e;
    slot_of[e] = v;
    stamp[v] = now;
    miss_e[r] = e;
    miss_s[r] = v;
  }
  __syncthreads();
  for (int a = tid; a < A; a += 1024) {
    const int ex = ids[a] - e0;
    slot_ids[a] = (ex >= 0 && ex < E) ? max(slot_of[ex], 0) : S + 1;  // S + 1: not this rank's expert
  }
  if (tid == 0) {
    miss_count[0] = nmiss;
    clock[0] = now;
    int hits = 0;
    for (int k = 0; k < E; ++k) hits += need[k];
    counters[0] += hits - nmiss;
    counters[1] += nmiss;
  }
}

struct CopyRegions {
  const uint8_t* src[6];
  uint8_t* dst[6];
  int64_t bytes[6];  // per expert
  int n;
};

__global__ void expert_copy_kernel(CopyRegions cr, const int32_t* __restrict__ miss_e, const int32_t* __restrict__ miss_s,
                                   const int32_t* __restrict__ miss_count, int64_t chunk) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  if (m >= *miss_count) return;
  const int64_t e = miss_e[m], s = miss_s[m];
  for (int r = 0; r < cr.n; ++r) {
    const int64_t nb = cr.bytes[r];
    const int64_t b0 = (int64_t)blockIdx.y * chunk, b1 = min(nb, b0 + chunk);
    const uint4* src = reinterpret_cast<const uint4*>(cr.src[r] + e * nb);
    uint4* dst = reinterpret_cast<uint4*>(cr.dst[r] + s * nb);
    for (int64_t i = b0 / 16 + threadIdx.x; i < b1 / 16; i += blockDim.x) dst[i] = src[i];
  }
}

void lru_route(torch::Tensor ids, int64_t e0, int64_t E, int64_t S, torch::Tensor slot_of, torch::Tensor expert_of,
               torch::Tensor stamp, torch::Tensor clock, torch::Tensor miss_e, torch::Tensor miss_s,
               torch::Tensor miss_count, torch::Tensor counters, torch::Tensor slot_ids, torch::Tensor status) {
  TORCH_CHECK(E <= LRU_MAX && S <= LRU_MAX && S >= 1, "lru_route: at most 1024 experts / slots");
  const at::cuda::CUDAGuard guard(ids.device());
  TORCH_CHECK(launch_pdl(lru_route_kernel, dim3(1), dim3(1024), 0, at::cuda::getCurrentCUDAStream(),
                         ids.data_ptr<int32_t>(), (int)ids.numel(), (int)e0, (int)E, (int)S,
                         slot_of.data_ptr<int32_t>(), expert_of.data_ptr<int32_t>(), stamp.data_ptr<int64_t>(),
                         clock.data_ptr<int64_t>(), miss_e.data_ptr<int32_t>(), miss_s.data_ptr<int32_t>(),
                         miss_count.data_ptr<int32_t>(), counters.data_ptr<int64_t>(), slot_ids.data_ptr<int32_t>(),
                         status.data_ptr<int>()) == cudaSuccess,
              "lru_route launch");
}

// srcs: pinned host uint8 tensors [E * bytes_per_expert]; dsts: device uint8 tensors [S * bytes_per_expert]
void expert_copy(std::vector<torch::Tensor> srcs, std::vector<torch::Tensor> dsts, std::vector<int64_t> bytes,
                 torch::Tensor miss_e, torch::Tensor miss_s, torch::Tensor miss_count, int64_t max_misses) {
  TORCH_CHECK(srcs.size() == dsts.size() && srcs.size() == bytes.size() && srcs.size() <= 6, "expert_copy: regions");
  CopyRegions cr = {};
  cr.n = (int)srcs.size();
  int64_t maxb = 0;
  for (int i = 0; i < cr.n; ++i) {
    TORCH_CHECK(srcs[i].is_pinned() && bytes[i] % 16 == 0, "expert_copy: pinned sources, 16-byte expert blocks");
    void* dp = nullptr;
    TORCH_CHECK(cudaHostGetDevicePointer(&dp, srcs[i].data_ptr(), 0) == cudaSuccess, "expert_copy: host mapping");
    cr.src[i] = reinterpret_cast<const uint8_t*>(dp);
    cr.dst[i] = dsts[i].data_ptr<uint8_t>();
    cr.bytes[i] = bytes[i];
    maxb = std::max(maxb, bytes[i]);
  }
  if (max_misses <= 0) return;
  const int64_t chunk = 64 * 1024;
  const at::cuda::CUDAGuard guard(miss_e.device());
  TORCH_CHECK(launch_pdl(expert_copy_kernel, dim3((unsigned)max_misses, (unsigned)((maxb + chunk - 1) / chunk)), dim3(256), 0,
                         at::cuda::getCurrentCUDAStream(), cr, miss_e.data_ptr<int32_t>(), miss_s.data_ptr<int32_t>(),
                         miss_count.data_ptr<int32_t>(), chunk) == cudaSuccess,
              "expert_copy launch");
}

}  // namespace r9k
