// Host-resident embedding tables: row gathers from pinned host memory through its unified (UVA)
// address, for tables too large for HBM -- the Flash-Next per-layer / n-gram embedding tables in
// fused int6 rows and the DeepSeek Engram tables in e4m3 with ue8m0 block scales.
//
// Row formats (bytes per row):
//   int6: dim codes in [-31, 31] stored + 32, four per 24-bit little-endian word (code i of a word =
//         (w >> 6 i) & 63), then one fp16 scale per 32 elements (reference: kernels/r9k_ple.hip:4-11,
//         the int6 GPTQ checkpoint format it serves);
//   fp8:  dim e4m3 bytes, then one ue8m0 exponent byte per 32 elements (value = e4m3 * 2^(e - 127)).
// One warp per row: lanes issue independent loads (a row is a few hundred bytes; PCIe / C2C latency
// dominates, so many rows must be in flight at once: the grid has one warp per requested row).
// Out-of-range ids produce zero rows instead of a host page fault.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp8.h>
#include "common.cuh"

namespace r9k {

template <int FMT>  // 0 int6, 1 fp8
__global__ void host_gather_kernel(const uint8_t* __restrict__ table, int64_t rows, int row_bytes, int dim,
                                   const int64_t* __restrict__ ids, int64_t n, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  const int64_t id = ids[warp];
  __nv_bfloat16* o = out + warp * dim;
  if (id < 0 || id >= rows) {
    for (int i = lane; i < dim; i += 32) o[i] = __float2bfloat16(0.f);
    return;
  }
  const uint8_t* row = table + id * (int64_t)row_bytes;
  if constexpr (FMT == 0) {
    const int words = dim / 4;
    const uint8_t* sc = row + dim * 6 / 8;
    for (int w = lane; w < words; w += 32) {
      const uint8_t* p = row + 3 * w;
      const uint32_t word = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16);
      const int g = (4 * w) / 32;
      const float s = __half2float(__ushort_as_half((unsigned short)(sc[2 * g] | (sc[2 * g + 1] << 8))));
#pragma unroll
      for (int k = 0; k < 4; ++k) o[4 * w + k] = __float2bfloat16((float)((int)((word >> (6 * k)) & 63u) - 32) * s);
    }
  } else {
    const uint8_t* sc = row + dim;
    for (int i = lane; i < dim; i += 32) {
      __nv_fp8_e4m3 v;
      v.__x = row[i];
      const int e = (int)sc[i / 32] - 127;
      o[i] = __float2bfloat16(float(v) * exp2f((float)e));
    }
  }
}

// table: CPU tensor in pinned memory (uint8 [rows, row_bytes]); ids: device int64 [n]; out: device bf16 [n, dim]
void host_gather(torch::Tensor table, torch::Tensor ids, int64_t fmt, int64_t dim, torch::Tensor out) {
  const int64_t n = ids.numel();
  if (n == 0) return;
  TORCH_CHECK(table.is_pinned() && table.dtype() == torch::kUInt8 && table.dim() == 2 && table.is_contiguous(),
              "host_gather: table must be a contiguous pinned uint8 [rows, row_bytes] CPU tensor");
  TORCH_CHECK(dim % 32 == 0, "host_gather: dim % 32");
  const int64_t rb = table.size(1);
  TORCH_CHECK(fmt == 0 ? rb == dim * 6 / 8 + dim / 32 * 2 : rb == dim + dim / 32, "host_gather: row bytes do not match the format");
  TORCH_CHECK(ids.is_cuda() && ids.dtype() == torch::kInt64 && out.is_cuda() && out.size(-1) == dim, "host_gather: ids / out");
  const at::cuda::CUDAGuard guard(ids.device());
  void* dptr = nullptr;
  TORCH_CHECK(cudaHostGetDevicePointer(&dptr, table.data_ptr(), 0) == cudaSuccess && dptr != nullptr,
              "host_gather: table is not mapped into the device address space");
  const dim3 grid((unsigned)((n * 32 + 255) / 256));
  auto st = at::cuda::getCurrentCUDAStream();
  auto kern = fmt == 0 ? host_gather_kernel<0> : host_gather_kernel<1>;
  TORCH_CHECK(launch_pdl(kern, grid, dim3(256), 0, st, reinterpret_cast<const uint8_t*>(dptr), table.size(0), (int)rb,
                         (int)dim, ids.data_ptr<int64_t>(), n, reinterpret_cast<__nv_bfloat16*>(out.data_ptr())) ==
                  cudaSuccess,
              "host_gather launch");
}

}  // namespace r9k
