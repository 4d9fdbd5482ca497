// EXL3-style trellis weights (3-bit class experts of DeepSeek-V4-class models): tile decode, full
// dequantisation (prefill: feeds the bf16 tcgen05 GEMM) and the decode-width GEMV.
//
// Format and decode (defined with a CPU oracle in quant/exl3.py): a linear [in -> out] is int16
// trellis [in/16, out/16, 16K] (one 16 x 16 tile per 256 weights, K bits each), f16 suh [in], f16 svh
// [out]; y = had(had(x * suh) @ W') * svh with the normalised 128-point Walsh-Hadamard transform.
// Weight i of a tile is the codebook value of the 16-bit window ending at bit (i + 1) K of the tile's
// circular bitstream (word w's bit 15 first). Codebooks: mcg (x = s * 0xCBAC1FED; (x & 0x8FFF8FFF) ^
// 0x3B603B60 read as two halves and summed) and mul1 (x = s * 0x83DCD12D; byte sum b; fma(1024 + b,
// h(0x1EEE), h(0xC931))). Weight i sits at tile row i / 16, column i % 16.
// (reference: kernels/r9k_exl3_gemv.hip, kernels/r9k_moe_exl3.hip -- which carry exllamav3's RDNA code;
// this file is an independent CUDA implementation of the decode from the format description.)
//
// Kernels
//   exl3_dequant_kernel: one CTA per 128 x 128 block: decode 64 tiles into smem (fp32), Walsh-Hadamard
//     along both dims, scale by suh / svh, store W_eff^T [out, in] bf16 (the GEMM's weight layout).
//   exl3_gemv_kernel<MR, CPW>: decode-width y' partials. grid (out / 128, ksplit, work items); the CTA
//     rotates its rows' input chunk (x * suh, Walsh-Hadamard per 128) into smem, then each warp walks the
//     tiles of one 16-column strip of the chunk: the warp stages a tile's words in smem, every lane
//     decodes CPW weights of one row per pass and accumulates them into MR x CPW fp32 registers (one
//     decode feeds every row). Lanes sharing a column set reduce with shuffles; partials go to scratch.
//     With a work list (MoE), work item z = (expert, first row, rows) selects the expert's matrix and
//     the rows; CTAs past the device-side count exit.
//   exl3_finish_kernel: sums the ksplit partials in order, Walsh-Hadamard per 128 outputs, * svh;
//     optionally SwiGLU of a gate/up pair; bf16 or fp32 out.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp16.h>
#include "common.cuh"

namespace r9k {

namespace {

R9K_DEVINL uint32_t tile_state(const uint16_t* words, int nwords, int i, int K) {
  const int nb = nwords * 16;
  int p = (i + 1) * K - 16;
  if (p < 0) p += nb;
  const int w = p >> 4, o = p & 15;
  const uint32_t v = ((uint32_t)words[w] << 16) | (uint32_t)words[(w + 1 == nwords) ? 0 : w + 1];
  return (v >> (16 - o)) & 0xFFFFu;
}

template <int CB>
R9K_DEVINL float codebook(uint32_t s) {
  if constexpr (CB == 1) {
    uint32_t x = s * 0xCBAC1FEDu;
    x = (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
    const float v = __half2float(__ushort_as_half((unsigned short)(x & 0xFFFFu))) +
                    __half2float(__ushort_as_half((unsigned short)(x >> 16)));
    return __half2float(__float2half_rn(v));
  } else {
    const uint32_t x = s * 0x83DCD12Du;
    const uint32_t b = (x & 0xFFu) + ((x >> 8) & 0xFFu) + ((x >> 16) & 0xFFu) + (x >> 24);
    const __half r = __hfma(__float2half_rn((float)(1024u + b)), __ushort_as_half((unsigned short)0x1EEE),
                            __ushort_as_half((unsigned short)0xC931));
    return __half2float(r);
  }
}

// in-place normalised 128-point Walsh-Hadamard transform of v[0..127] with stride `st`, by the 128
// threads t = 0..127 of a (sub)group that call it together (bar: a barrier over exactly those threads)
template <typename Bar>
R9K_DEVINL void wht128(float* v, int st, int t, Bar bar) {
#pragma unroll
  for (int h = 1; h < 128; h <<= 1) {
    float a = 0.f, b = 0.f;
    const int blk = t / h, off = t % h;
    const int i0 = (blk * 2) * h + off;
    if (t < 64) {
      a = v[i0 * st];
      b = v[(i0 + h) * st];
    }
    bar();
    if (t < 64) {
      v[i0 * st] = a + b;
      v[(i0 + h) * st] = a - b;
    }
    bar();
  }
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// full dequantisation: W_eff^T [out, in] bf16
// ------------------------------------------------------------------------------------------------
template <int CB>
__global__ void __launch_bounds__(256) exl3_dequant_kernel(const uint16_t* __restrict__ trellis, int K,
                                                          const __half* __restrict__ suh, const __half* __restrict__ svh,
                                                          int n_in, int n_out, __nv_bfloat16* __restrict__ out) {
  // no early trigger: the output is a GEMM weight, and the GEMM requests its first weight tiles
  // before its own grid-dependency wait, so it must not start until this grid has finished
  pdl_wait();
  extern __shared__ float sw[];  // [128][129]
  const int ob = blockIdx.x, ib = blockIdx.y, tid = threadIdx.x;
  const int nw = 16 * K, to_n = n_out / 16;
  // decode: 64 tiles (8 x 8), 256 weights each
  for (int e = tid; e < 128 * 128; e += 256) {
    const int tile = e >> 8, i = e & 255;
    const int a = ib * 8 + (tile >> 3), b = ob * 8 + (tile & 7);
    const uint16_t* words = trellis + ((int64_t)a * to_n + b) * nw;
    const float v = codebook<CB>(tile_state(words, nw, i, K));
    sw[((tile >> 3) * 16 + (i >> 4)) * 129 + (tile & 7) * 16 + (i & 15)] = v;
  }
  __syncthreads();
  // rows (input dim) transform for each output column: two half-blocks of 128 threads handle 64 columns each
  const int half = tid >> 7, t = tid & 127;
  auto bar = [] { __syncthreads(); };
  for (int c = 0; c < 64; ++c) wht128(sw + (half * 64 + c), 129, t, bar);
  for (int r = 0; r < 64; ++r) wht128(sw + (half * 64 + r) * 129, 1, t, bar);
  for (int e = tid; e < 128 * 128; e += 256) {
    const int o = e >> 7, i = e & 127;  // out row, in column (coalesced along in)
    const int gi = ib * 128 + i, go = ob * 128 + o;
    const float v = sw[i * 129 + o] * __half2float(suh[gi]) * __half2float(svh[go]) * (1.f / 128.f);
    out[(int64_t)go * n_in + gi] = __float2bfloat16(v);
  }
}

// ------------------------------------------------------------------------------------------------
// decode-width GEMV partials
// ------------------------------------------------------------------------------------------------
struct Exl3Gemv {
  const uint16_t* trellis;  // expert 0; expert e at + e * t_stride
  int64_t t_stride;
  const __half* suh;  // [in] (+ e * n_in)
  const __half* svh;
  const __nv_bfloat16* x;  // rows [*, ldx]
  int64_t ldx;
  float* part;  // [ksplit][work][MR][out]
  int n_in, n_out, K, ksplit, chunk, M;
  const int32_t* work;  // (expert, row0, rows) or null: single matrix, rows 0..M-1
  const int32_t* work_count;
};

template <int CB, int MR, int CPW>
__global__ void __launch_bounds__(256) exl3_gemv_kernel(const Exl3Gemv g) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float xs[];  // [MR][chunk]
  __shared__ uint16_t tw[8][16 * 8];
  const int z = blockIdx.z;
  int e = 0, row0 = 0, rows = g.M;
  if (g.work != nullptr) {
    if (z >= *g.work_count) return;
    e = g.work[3 * z];
    row0 = g.work[3 * z + 1];
    rows = min(g.work[3 * z + 2], MR);
  }
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k0 = blockIdx.y * g.chunk;
  const __half* suh = g.suh + (int64_t)e * g.n_in;
  // input rotation of this chunk: xs[m][k] = had(x * suh)
  for (int idx = tid; idx < MR * g.chunk; idx += 256) {
    const int m = idx / g.chunk, k = idx % g.chunk;
    xs[idx] = (m < rows) ? __bfloat162float(g.x[(int64_t)(row0 + m) * g.ldx + k0 + k]) * __half2float(suh[k0 + k]) : 0.f;
  }
  __syncthreads();
  {
    auto bar = [] { __syncthreads(); };
    const int half = tid >> 7, t = tid & 127;
    const int nblk = MR * (g.chunk / 128);  // even: MR is 8 or 16
    // blocks are transformed by the two 128-thread halves in lockstep; both halves run every step
    for (int base = 0; base < nblk; base += 2) {
      const int bidx = base + half;
      float* v = xs + (bidx < nblk ? bidx * 128 : 0);
      // threads of a half whose block does not exist still take part in the barriers
      float a = 0.f, b = 0.f;
#pragma unroll 1
      for (int h = 1; h < 128; h <<= 1) {
        const int blk = t / h, off = t % h, i0 = (blk * 2) * h + off;
        if (t < 64 && bidx < nblk) {
          a = v[i0];
          b = v[i0 + h];
        }
        bar();
        if (t < 64 && bidx < nblk) {
          v[i0] = a + b;
          v[i0 + h] = a - b;
        }
        bar();
      }
    }
  }
  const float rs = 0.08838834764831845f;  // 1 / sqrt(128)
  // each warp: one 16-column strip of this CTA's 128 outputs
  constexpr int LPR = 16 / CPW;   // lanes per tile row
  constexpr int RPP = 32 / LPR;   // tile rows per pass
  constexpr int PASSES = 16 / RPP;
  const int col0 = (lane % LPR) * CPW;
  const int strip = blockIdx.x * 8 + warp;
  const int nw = 16 * g.K;
  const uint16_t* tbase = g.trellis + (int64_t)e * g.t_stride;
  float acc[MR][CPW];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int j = 0; j < CPW; ++j) acc[m][j] = 0.f;
  const int to_n = g.n_out / 16;
  for (int a = k0 / 16; a < (k0 + g.chunk) / 16; ++a) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(tbase + ((int64_t)a * to_n + strip) * nw);
    __syncwarp();
    if (lane < nw / 2) reinterpret_cast<uint32_t*>(tw[warp])[lane] = src[lane];
    __syncwarp();
#pragma unroll
    for (int ps = 0; ps < PASSES; ++ps) {
      const int r = lane / LPR + ps * RPP;
      const int kk = a * 16 + r - k0;
      float w[CPW];
#pragma unroll
      for (int j = 0; j < CPW; ++j) w[j] = codebook<CB>(tile_state(tw[warp], nw, r * 16 + col0 + j, g.K));
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const float xv = xs[m * g.chunk + kk] * rs;
#pragma unroll
        for (int j = 0; j < CPW; ++j) acc[m][j] = fmaf(xv, w[j], acc[m][j]);
      }
    }
  }
  // reduce over lanes that share col0 (lane % LPR)
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int j = 0; j < CPW; ++j) {
      float v = acc[m][j];
#pragma unroll
      for (int o = LPR; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[m][j] = v;
    }
  if (lane < LPR) {
    const int nz = gridDim.z;
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      if (m < rows) {
        float* dst = g.part + (((int64_t)blockIdx.y * nz + z) * MR + m) * g.n_out + strip * 16 + col0;
#pragma unroll
        for (int j = 0; j < CPW; ++j) dst[j] = acc[m][j];
      }
    }
  }
}

// out rows: y[row0 + m][o] = svh[o] * had(sum_s part[s][z][m]) (+ SwiGLU of a gate / up pair)
template <bool SWIGLU>
__global__ void __launch_bounds__(128) exl3_finish_kernel(const float* __restrict__ part, const float* __restrict__ part_up,
                                                          const __half* __restrict__ svh, const __half* __restrict__ svh_up,
                                                          int ksplit, int nz, int MR, int n_out, const int32_t* __restrict__ work,
                                                          const int32_t* __restrict__ work_count, int M,
                                                          void* __restrict__ out, int64_t ldo, int out_f32) {
  pdl_wait();
  pdl_trigger();
  __shared__ float v[128], u[128];
  const int ob = blockIdx.x, m = blockIdx.y, z = blockIdx.z, t = threadIdx.x;
  int e = 0, row0 = 0, rows = M;
  if (work != nullptr) {
    if (z >= *work_count) return;
    e = work[3 * z];
    row0 = work[3 * z + 1];
    rows = min(work[3 * z + 2], MR);
  }
  if (m >= rows) return;
  const int o = ob * 128 + t;
  float s = 0.f, su = 0.f;
  for (int k = 0; k < ksplit; ++k) {
    const int64_t idx = (((int64_t)k * nz + z) * MR + m) * n_out + o;
    s += part[idx];
    if (SWIGLU) su += part_up[idx];
  }
  v[t] = s;
  u[t] = su;
  __syncthreads();
  auto bar = [] { __syncthreads(); };
  wht128(v, 1, t, bar);
  if (SWIGLU) wht128(u, 1, t, bar);
  const float rs = 0.08838834764831845f;
  float y = v[t] * rs * __half2float(svh[(int64_t)e * n_out + o]);
  if (SWIGLU) {
    const float up = u[t] * rs * __half2float(svh_up[(int64_t)e * n_out + o]);
    y = y / (1.f + __expf(-y)) * up;
  }
  if (out_f32) reinterpret_cast<float*>(out)[(int64_t)(row0 + m) * ldo + o] = y;
  else reinterpret_cast<__nv_bfloat16*>(out)[(int64_t)(row0 + m) * ldo + o] = __float2bfloat16(y);
}

// ------------------------------------------------------------------------------------------------
void exl3_dequant(torch::Tensor trellis, torch::Tensor suh, torch::Tensor svh, int64_t K, int64_t cb, torch::Tensor out) {
  const int64_t n_in = trellis.size(0) * 16, n_out = trellis.size(1) * 16;
  TORCH_CHECK(trellis.size(2) == 16 * K && trellis.is_contiguous() && K >= 1 && K <= 8, "exl3: trellis [in/16, out/16, 16K]");
  TORCH_CHECK(n_in % 128 == 0 && n_out % 128 == 0, "exl3: in and out must be multiples of 128");
  TORCH_CHECK(out.size(0) == n_out && out.size(1) == n_in && out.dtype() == torch::kBFloat16, "exl3_dequant: out [out, in] bf16");
  const at::cuda::CUDAGuard guard(trellis.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const size_t smem = 128 * 129 * sizeof(float);
  auto kern = cb == 1 ? exl3_dequant_kernel<1> : exl3_dequant_kernel<2>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  TORCH_CHECK(launch_pdl(kern, dim3((unsigned)(n_out / 128), (unsigned)(n_in / 128)), dim3(256), smem, st,
                         reinterpret_cast<const uint16_t*>(trellis.data_ptr()), (int)K,
                         reinterpret_cast<const __half*>(suh.data_ptr()), reinterpret_cast<const __half*>(svh.data_ptr()),
                         (int)n_in, (int)n_out, reinterpret_cast<__nv_bfloat16*>(out.data_ptr())) == cudaSuccess,
              "exl3_dequant launch");
}

// y partials: x [rows, in] bf16; trellis [E?][in/16, out/16, 16K]; part [ksplit * nz * MR * out] f32.
void exl3_gemv(torch::Tensor trellis, torch::Tensor suh, int64_t K, int64_t cb, torch::Tensor x, int64_t M,
               c10::optional<torch::Tensor> work, c10::optional<torch::Tensor> work_count, int64_t nz, int64_t ksplit,
               torch::Tensor part) {
  const bool stacked = trellis.dim() == 4;
  const int64_t ti = trellis.size(stacked ? 1 : 0), to = trellis.size(stacked ? 2 : 1);
  const int64_t n_in = ti * 16, n_out = to * 16;
  TORCH_CHECK(trellis.size(stacked ? 3 : 2) == 16 * K && trellis.is_contiguous(), "exl3_gemv: trellis shape");
  TORCH_CHECK(n_in % (128 * ksplit) == 0 && n_out % 128 == 0, "exl3_gemv: in must split into 128-multiples");
  TORCH_CHECK(x.dtype() == torch::kBFloat16 && x.stride(1) == 1 && x.size(1) == n_in, "exl3_gemv: x [rows, in] bf16");
  const int MR = M <= 8 ? 8 : 16;
  TORCH_CHECK(M >= 1 && M <= 16, "exl3_gemv: 1..16 rows per matrix");
  TORCH_CHECK(part.numel() >= ksplit * nz * MR * n_out, "exl3_gemv: partial scratch too small");
  const bool has_work = work.has_value() && work->defined();
  Exl3Gemv g;
  g.trellis = reinterpret_cast<const uint16_t*>(trellis.data_ptr());
  g.t_stride = stacked ? ti * to * 16 * K : 0;
  g.suh = reinterpret_cast<const __half*>(suh.data_ptr());
  g.svh = nullptr;
  g.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  g.ldx = x.stride(0);
  g.part = part.data_ptr<float>();
  g.n_in = (int)n_in; g.n_out = (int)n_out; g.K = (int)K; g.ksplit = (int)ksplit; g.chunk = (int)(n_in / ksplit);
  g.M = (int)M;
  g.work = has_work ? work->data_ptr<int32_t>() : nullptr;
  g.work_count = has_work ? work_count->data_ptr<int32_t>() : nullptr;
  const at::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const size_t smem = (size_t)MR * g.chunk * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "exl3_gemv: input chunk too large; raise ksplit");
  const dim3 grid((unsigned)(n_out / 128), (unsigned)ksplit, (unsigned)nz);
#define R9K_EXL3_GEMV(CBV, MRV, CPWV)                                                                  \
  {                                                                                                    \
    auto kern = exl3_gemv_kernel<CBV, MRV, CPWV>;                                                      \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                \
    TORCH_CHECK(launch_pdl(kern, grid, dim3(256), smem, st, g) == cudaSuccess, "exl3_gemv launch");    \
  }
  if (cb == 1) {
    if (MR == 8) R9K_EXL3_GEMV(1, 8, 8) else R9K_EXL3_GEMV(1, 16, 4)
  } else {
    if (MR == 8) R9K_EXL3_GEMV(2, 8, 8) else R9K_EXL3_GEMV(2, 16, 4)
  }
#undef R9K_EXL3_GEMV
}

void exl3_finish(torch::Tensor part, c10::optional<torch::Tensor> part_up, torch::Tensor svh,
                 c10::optional<torch::Tensor> svh_up, int64_t ksplit, int64_t nz, int64_t M, int64_t n_out,
                 c10::optional<torch::Tensor> work, c10::optional<torch::Tensor> work_count, torch::Tensor out) {
  const int MR = M <= 8 ? 8 : 16;
  const bool has_work = work.has_value() && work->defined();
  const bool sw = part_up.has_value() && part_up->defined();
  const at::cuda::CUDAGuard guard(part.device());
  auto st = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(out.stride(1) == 1 && out.size(1) == n_out && n_out % 128 == 0, "exl3_finish: out [rows, out]");
  const dim3 grid((unsigned)(n_out / 128), (unsigned)MR, (unsigned)nz);
  const int of32 = out.dtype() == torch::kFloat32 ? 1 : 0;
  auto kern = sw ? exl3_finish_kernel<true> : exl3_finish_kernel<false>;
  TORCH_CHECK(launch_pdl(kern, grid, dim3(128), 0, st, part.data_ptr<float>(), sw ? part_up->data_ptr<float>() : nullptr,
                         reinterpret_cast<const __half*>(svh.data_ptr()),
                         sw ? reinterpret_cast<const __half*>(svh_up->data_ptr()) : nullptr, (int)ksplit, (int)nz, MR,
                         (int)n_out, has_work ? work->data_ptr<int32_t>() : nullptr,
                         has_work ? work_count->data_ptr<int32_t>() : nullptr, (int)M, out.data_ptr(), out.stride(0),
                         of32) == cudaSuccess,
              "exl3_finish launch");
}

}  // namespace r9k
