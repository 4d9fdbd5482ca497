// Device-side view of the symmetric all-reduce regions (see comm.cu for the protocol).
//
// Region of every rank: [flags: 2 buffers x 8 sources x 256 tiles x u32 (16 KiB, padded to 64 KiB)]
//                       [data : 2 buffers x world sources x slot_elems bf16]
//                       [LL   : 2 buffers x world sources x slot_elems/2 {bf16x2, u32 epoch} pairs]
// Call g (global index = step * calls_per_step + k) uses buffer g & 1 and epoch g + 1.
//
// LL ("low-latency") slots carry the call's epoch inside every 8-byte word next to two bf16 values,
// so a reader knows a word has arrived by its epoch alone: no fence, no separate flag, no round trip
// before the data moves. A 16-byte store writes two such words; readers check both epochs (each
// aligned 8-byte half is written as one unit).
#pragma once
#include <torch/extension.h>
#include "common.cuh"

namespace r9k {

constexpr int AR_MAX_WORLD = 8;
constexpr int AR_MAX_TILES = 256;
constexpr int64_t AR_FLAG_BYTES = 64 * 1024;

struct ArPeers {
  uint8_t* base[AR_MAX_WORLD];  // region of every rank, mapped into this process
  int rank;
  int world;
  int calls_per_step;
  int64_t slot_elems;
  const uint32_t* step;  // this rank's device step counter
};

R9K_DEVINL uint32_t ar_global_call(const ArPeers& pe, int call) {
  return (uint32_t)(*pe.step) * (uint32_t)pe.calls_per_step + (uint32_t)call;
}
R9K_DEVINL uint32_t ar_epoch(const ArPeers& pe, int call) { return ar_global_call(pe, call) + 1u; }

R9K_DEVINL __nv_bfloat16* ar_slot(const ArPeers& pe, int p, int call, int src) {
  const uint32_t b = ar_global_call(pe, call) & 1u;
  return reinterpret_cast<__nv_bfloat16*>(pe.base[p] + AR_FLAG_BYTES) + ((int64_t)b * pe.world + src) * pe.slot_elems;
}
R9K_DEVINL uint32_t* ar_flag_ptr(const ArPeers& pe, int p, int call, int src, int tile) {
  const uint32_t b = ar_global_call(pe, call) & 1u;
  return reinterpret_cast<uint32_t*>(pe.base[p]) + ((int64_t)b * AR_MAX_WORLD + src) * AR_MAX_TILES + tile;
}

R9K_DEVINL uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
R9K_DEVINL void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
R9K_DEVINL uint4 ld_volatile_u4(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}

// LL slot of source `src` in rank p's region, buffer `buf`: u32 words, element e of row t at word
// (t * H + e) rounded down to even, its pair's epoch at the next word (slot = slot_elems words).
R9K_DEVINL uint32_t* ar_ll_slot(const ArPeers& pe, int p, uint32_t buf, int src) {
  uint8_t* ll = pe.base[p] + AR_FLAG_BYTES + 2 * (int64_t)pe.world * pe.slot_elems * 2;
  return reinterpret_cast<uint32_t*>(ll) + ((int64_t)buf * pe.world + src) * pe.slot_elems;
}
R9K_DEVINL void st_ll16(uint32_t* p, uint32_t d0, uint32_t d1, uint32_t e) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(d0), "r"(e), "r"(d1), "r"(e)
               : "memory");
}
R9K_DEVINL uint4 ld_ll16(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p) : "memory");
  return v;
}

// Raise tile `tile`'s flag for this rank's contribution in every rank's region. Called by one thread
// after a CTA barrier that orders every writer's data stores before it: the system-scope fence plus
// the release store make those (cumulatively ordered) stores visible before the flag.
R9K_DEVINL void ar_raise_flags(const ArPeers& pe, int call, int tile, uint32_t epoch) {
  __threadfence_system();
  for (int p = 0; p < pe.world; ++p) st_release_sys(ar_flag_ptr(pe, p, call, pe.rank, tile), epoch);
}

// Resolved once per kernel: this call's epoch and the destination slot of this rank in every region.
struct ArCall {
  uint32_t epoch;
  __nv_bfloat16* dst[AR_MAX_WORLD];
};
R9K_DEVINL ArCall ar_resolve(const ArPeers& pe, int call) {
  ArCall c;
  const uint32_t g = ar_global_call(pe, call);
  c.epoch = g + 1u;
  const uint32_t b = g & 1u;
#pragma unroll
  for (int p = 0; p < AR_MAX_WORLD; ++p)
    c.dst[p] = p < pe.world ? reinterpret_cast<__nv_bfloat16*>(pe.base[p] + AR_FLAG_BYTES) +
                                  ((int64_t)b * pe.world + pe.rank) * pe.slot_elems
                            : nullptr;
  return c;
}

inline ArPeers make_peers(const torch::Tensor& peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t H,
                          const torch::Tensor& step, int64_t calls_per_step = 2) {
  TORCH_CHECK(world >= 1 && world <= AR_MAX_WORLD, "all-reduce world size must be 1..8");
  TORCH_CHECK(peers.numel() >= world && peers.dtype() == torch::kInt64 && peers.device().is_cpu(),
              "peer pointer table: int64 CPU tensor");
  TORCH_CHECK(H / 128 <= AR_MAX_TILES, "hidden too large for the flag table");
  TORCH_CHECK(calls_per_step % 2 == 0, "calls per step must be even so buffers alternate across steps");
  ArPeers pe = {};
  const int64_t* pp = peers.data_ptr<int64_t>();
  for (int i = 0; i < world; ++i) pe.base[i] = reinterpret_cast<uint8_t*>(pp[i]);
  pe.rank = (int)rank;
  pe.world = (int)world;
  pe.calls_per_step = (int)calls_per_step;
  pe.slot_elems = slot_elems;
  pe.step = reinterpret_cast<const uint32_t*>(step.data_ptr());
  return pe;
}

}  // namespace r9k
