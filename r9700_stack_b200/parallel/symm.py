"""Symmetric-memory tensor-parallel communicator with the all-reduce fused into its neighbours.

Each rank allocates one device region (CUDA IPC shared with its peers). For decode-sized batches
(``R9K_AR_MODE``):

* ``ll`` (default): the row-parallel GEMM that ends a sublayer (o_proj, GDN out_proj, FFN
  down_proj) runs with the push epilogue (``gemm_mx_push``, LL form): its bf16 partial tiles go
  straight into every rank's LL slot over NVLink with the call's epoch inside every 8-byte word;
  other producers use ``ll_push``. The RMSNorm that follows runs as ``ar_ll_rmsnorm``: it polls its
  own region until every source's words carry the epoch, sums the partials in rank order
  (bit-identical on every rank), adds the residual and emits the next GEMM's MXFP8 input. The data
  is its own ready signal: no fence and no flag round trip (the release/acquire flag handshake costs
  two system-scope releases, ~5.6 us a round trip on B200 against ~2.5 us relaxed;
  ``tuning/arbench.py --latency``).
* ``pull``: the GEMM writes its partial locally; the consumer raises a ready flag and reads the
  peers' partials over NVLink.
* ``push``: as ``ll`` but plain bf16 slots with per-tile flags (fence + release store).

No separate all-reduce kernel runs for decode. Batches larger than the slot (prefill) go through the
NVLS two-shot all-reduce (``parallel.nvls``: the switch reduces, every element once, same bits on
every rank; ``R9K_PREFILL_AR``), and the logits all-gather through the NVLS all-gather
(``R9K_LOGITS_AG``); NCCL takes them where the platform has no multicast object.
Reference counterpart: the one-kernel P2P all-reduce family of r9700_vllm/comm/r9k_ar.py:87-601
(PCIe pair/quartet/host stages); on NVSwitch every peer is one hop, so there is no hierarchy.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _native
from ..utils import status as _status
from .comm import NcclComm

AR_FLAG_BYTES = 64 * 1024


class SymmComm(NcclComm):
    """NCCL communicator plus the fused push / reduce-norm path for up to ``max_tokens`` rows."""

    fused = True

    def __init__(self, hidden: int, max_tokens: int, calls_per_step: int, device, group=None,
                 timeout_s: float = 2.0, max_prefill_tokens: int = 8192):
        super().__init__(group)
        assert calls_per_step % 2 == 0
        self.device = torch.device(device)
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.calls_per_step = calls_per_step
        self.timeout_s = timeout_s
        self.slot_elems = max_tokens * hidden
        ops = _native.ops()
        # flag page, plain slots (pull / push), LL slots (two bf16 + an epoch per 8 bytes)
        nbytes = AR_FLAG_BYTES + 2 * self.world_size * self.slot_elems * 2 + 2 * self.world_size * self.slot_elems * 4
        # set-up is all-or-nothing: a rank that cannot allocate, export or open a region makes every
        # rank keep NCCL (reference: comm/r9k_ar.py:422-439, the "ok" exchange of every rank)
        self.local_ptr, self._opened, ok, handle = 0, [], True, b""
        try:
            self.local_ptr = int(ops.symm_alloc(nbytes))
            handle = ops.symm_ipc_handle(self.local_ptr).numpy().tobytes()
        except Exception as e:  # noqa: BLE001 - reported and agreed on below
            ok, self.setup_error = False, repr(e)
        handles = [None] * self.world_size
        if self.world_size > 1:
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles = [handle]
        ptrs = []
        if ok and all(handles):
            try:
                for i, h in enumerate(handles):
                    if i == self.rank:
                        ptrs.append(self.local_ptr)
                    else:
                        p = int(ops.symm_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
                        self._opened.append(p)
                        ptrs.append(p)
            except Exception as e:  # noqa: BLE001
                ok, self.setup_error = False, repr(e)
        else:
            ok = False
        if self.world_size > 1:
            flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
            ok = bool(int(flag))
        if not ok:
            import logging

            logging.getLogger("vllm.r9700_stack_b200").warning(
                "symmetric-memory set-up failed on some rank (%s): every rank keeps NCCL",
                getattr(self, "setup_error", "a peer"))
            self.fused = False  # the models then route every all-reduce through NCCL
            for p_ in self._opened:
                ops.symm_close(p_)
            self._opened = []
            if self.local_ptr:
                ops.symm_free(self.local_ptr)
                self.local_ptr = 0
            ptrs = [0] * self.world_size
        self.peers = torch.tensor(ptrs, dtype=torch.int64)
        self.step = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.barrier()
        # lossy compressed all-reduce for prefill-sized messages (opt-in: R9K_AR_QUANT_BITS=4|6)
        from .. import knobs

        # NVLS (multicast) collectives for prefill all-reduces and the logits all-gather
        self.nvls = None
        if self.world_size > 1 and (knobs.get("R9K_PREFILL_AR") == "symm" or knobs.get("R9K_LOGITS_AG") == "symm"):
            from .nvls import NvlsComm

            try:
                cap = max(max_prefill_tokens * hidden * 2, 64 << 20)
                nv = NvlsComm(self.device, group=group, capacity_bytes=(cap + (1 << 20) - 1) // (1 << 20) * (1 << 20),
                              timeout_s=timeout_s)
                self.nvls = nv if nv.available else None
            except Exception as e:  # noqa: BLE001 - no multicast support: NCCL keeps these collectives
                import logging

                logging.getLogger("vllm.r9700_stack_b200").info("NVLS unavailable (%s); NCCL for prefill", e)
        self._ag_out: dict = {}
        self.wht_bits = knobs.get_int("R9K_AR_QUANT_BITS") if self.world_size > 1 else 0
        self.wht_min_bytes = knobs.get_int("R9K_AR_QUANT_MIN_KB") * 1024
        self.wht = None
        if self.wht_bits in (4, 6):
            from .collectives import SymmCollectives

            chunks = -(-max_prefill_tokens * hidden // 4096)
            self.wht = SymmCollectives(self.device, group=group, slot_bytes=self.world_size * chunks * (64 * 8 * self.wht_bits + 128),
                                       timeout_s=timeout_s)

    # -------------------------------------------------------------------------------------------
    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        """Unfused all-reduce (prefill): the lossy compressed kernel when enabled, the NVLS two-shot
        kernel when the platform has multicast, else NCCL."""
        from .. import knobs

        if (self.wht is not None and t.numel() * t.element_size() >= self.wht_min_bytes
                and self.wht.wht_ok(t, self.wht_bits)):
            t.copy_(self.wht.all_reduce_wht(t, self.wht_bits))
            return t
        if self.nvls is not None and knobs.get("R9K_PREFILL_AR") == "symm" and self.nvls.fits_all_reduce(t):
            from ..utils.trace import note_all_reduce

            note_all_reduce(t.numel() * t.element_size())
            return self.nvls.all_reduce_(t)
        return super().all_reduce_(t)

    def all_gather_lastdim(self, t: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """[R, n] per rank -> [R, world * n]: the NVLS all-gather for fp32 logits, else NCCL."""
        from .. import knobs

        if (self.nvls is not None and knobs.get("R9K_LOGITS_AG") == "symm" and t.dim() == 2
                and t.is_contiguous() and self.nvls.fits_all_gather(t)):
            R, n = t.shape
            key = (R, n, t.dtype)
            buf = self._ag_out.get(key)
            if buf is None:
                buf = torch.empty(self.world_size, R, n, dtype=t.dtype, device=t.device)
                self._ag_out[key] = buf
            self.nvls.all_gather(t, buf)
            res = buf.permute(1, 0, 2).reshape(R, self.world_size * n)
            if out is not None:
                out.copy_(res)
                return out
            return res
        return super().all_gather_lastdim(t, out)

    def can_fuse(self, T: int) -> bool:
        return 0 < T <= self.max_tokens

    def step_begin(self) -> None:
        _native.ops().symm_step_begin(self.step)

    def gemm_push(self, act, w, call: int) -> None:
        _native.ops().gemm_mx_push(w.q, w.sf, w.fp4, act.q, act.sf, w.N, self.peers, self.rank, self.world_size,
                                   self.slot_elems, call, self.step, self.calls_per_step,
                                   _status.status(self.device), _gemm_ws(self.device), 1 if self.mode == "ll" else 0)

    @property
    def mode(self) -> str:
        from .. import knobs

        return knobs.get("R9K_AR_MODE") or "ll"

    def out_buffer(self, call: int, T: int) -> torch.Tensor:
        """Pull mode: where this rank's row-parallel GEMM writes its partial for call `call` (a static
        address per call site: buffer call % 2 of this rank's region)."""
        off = AR_FLAG_BYTES + (call & 1) * self.slot_elems * 2
        return _native.ops().symm_view(self.local_ptr, off, T, self.hidden, self.device.index or 0)

    def push(self, x: torch.Tensor, call: int) -> None:
        fn = _native.ops().ll_push if self.mode == "ll" else _native.ops().push_partial
        fn(x, self.peers, self.rank, self.world_size, self.slot_elems, call, self.step, self.calls_per_step)

    def ar_rmsnorm(self, call: int, T: int, w: torch.Tensor, eps: float, plus_one: bool, *, residual=None,
                   residual_out=None, y=None, quant_out=None) -> None:
        o = _native.ops()
        fn = {"pull": o.ar_pull_rmsnorm, "ll": o.ar_ll_rmsnorm}.get(self.mode, o.ar_rmsnorm)
        fn(self.peers, self.rank, self.world_size, self.slot_elems, call, self.step,
                                 self.calls_per_step, T, residual, residual_out, w, float(eps), bool(plus_one), y,
                                 quant_out.q if quant_out is not None else None,
                                 quant_out.sf if quant_out is not None else None,
                                 _status.status(self.device), float(self.timeout_s))

    def close(self) -> None:
        ops = _native.ops()
        self.nvls = None
        if self.wht is not None:
            self.wht.close()
            self.wht = None
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            ops.symm_close(p)
        self._opened = []
        if self.local_ptr:
            ops.symm_free(self.local_ptr)
            self.local_ptr = 0


def _gemm_ws(device):
    from ..ops.linear import gemm_workspace

    return gemm_workspace(device)
