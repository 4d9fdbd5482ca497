// NVLink latency probes between two ranks of the symmetric regions (tuning tools: they give the floor
// under every fused collective, so a fused kernel's time can be split into protocol and transfer).
//
//   p2p_pingpong  one thread per rank. Role 0 stores i into a word of the peer's region and waits for
//                 the answer i in its own region; role 1 waits, then answers. `iters` round trips in one
//                 kernel; mode 0 uses st.release.sys / ld.acquire.sys, mode 1 relaxed system-scope
//                 accesses, mode 2 relaxed accesses with a fence.sc.sys before every store (the
//                 publish pattern of a producer that wrote data first).
//   p2p_read      one thread issues `iters` dependent loads (each address depends on the previous
//                 value) from the peer's region: the NVLink load round trip.
// Every wait is bounded (status word on timeout). Both ranks launch the probe at the same time, one
// process per GPU, so the two spinning kernels always run concurrently.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace r9k {

R9K_DEVINL void st_word(uint32_t* p, uint32_t v, int mode) {
  if (mode == 0) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
  else {
    if (mode == 2) asm volatile("fence.sc.sys;" ::: "memory");
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
  }
}
R9K_DEVINL uint32_t ld_word(const uint32_t* p, int mode) {
  uint32_t v;
  if (mode == 0) asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  else asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void p2p_pingpong_kernel(uint32_t* mine, uint32_t* peer, int iters, int role, int mode,
                                    uint64_t timeout_ns, int* status, long long* out_ns) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  for (int i = 1; i <= iters && ok; ++i) {
    if (role == 0) st_word(peer, (uint32_t)i, mode);
    const uint64_t w0 = globaltimer_ns();
    while (ld_word(mine, mode) < (uint32_t)i) {
      if (globaltimer_ns() - w0 > timeout_ns) {
        report_error(status, kErrPeerTimeout, 900, i);
        ok = false;
        break;
      }
    }
    if (ok && role == 1) st_word(peer, (uint32_t)i, mode);
  }
  out_ns[0] = (long long)(globaltimer_ns() - t0);
}

__global__ void p2p_read_kernel(const uint32_t* peer, int iters, long long* out_ns, uint32_t* sink) {
  if (threadIdx.x != 0) return;
  uint32_t v = 0;
  const uint64_t t0 = globaltimer_ns();
  for (int i = 0; i < iters; ++i) v = ld_word(peer + (v & 1u), 1);  // address depends on the last value
  out_ns[0] = (long long)(globaltimer_ns() - t0);
  sink[0] = v;
}

// kind 0: ping-pong (mode as above), kind 1: dependent remote loads. Words at byte offset `off` of each
// region (reset by the caller). Returns the kernel's elapsed nanoseconds (int64 on the device).
torch::Tensor p2p_probe(torch::Tensor peers, int64_t rank, int64_t peer_rank, int64_t off, int64_t kind, int64_t mode,
                        int64_t iters, torch::Tensor status, double timeout_s) {
  TORCH_CHECK(peers.device().is_cpu() && peers.dtype() == torch::kInt64, "p2p_probe: CPU int64 peer table");
  TORCH_CHECK(rank != peer_rank && rank >= 0 && peer_rank >= 0 && rank < peers.numel() && peer_rank < peers.numel(),
              "p2p_probe: two distinct ranks");
  TORCH_CHECK(off % 64 == 0 && iters > 0, "p2p_probe: word offset 64-byte aligned, iters > 0");
  const int64_t* pp = peers.data_ptr<int64_t>();
  uint32_t* mine = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(pp[rank]) + off);
  uint32_t* peer = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(pp[peer_rank]) + off);
  auto out = torch::zeros({2}, torch::dtype(torch::kInt64).device(status.device()));
  const at::cuda::CUDAGuard guard(status.device());
  auto st = at::cuda::getCurrentCUDAStream();
  if (kind == 0) {
    const int role = rank < peer_rank ? 0 : 1;
    p2p_pingpong_kernel<<<1, 32, 0, st>>>(mine, peer, (int)iters, role, (int)mode, (uint64_t)(timeout_s * 1e9),
                                          status.data_ptr<int>(), reinterpret_cast<long long*>(out.data_ptr<int64_t>()));
  } else {
    p2p_read_kernel<<<1, 32, 0, st>>>(peer, (int)iters, reinterpret_cast<long long*>(out.data_ptr<int64_t>()),
                                      reinterpret_cast<uint32_t*>(out.data_ptr<int64_t>() + 1));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace r9k
