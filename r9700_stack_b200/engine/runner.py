"""Model runner: step metadata, CUDA graphs for decode, sampling.

Per step the host packs every int32 metadata field into one pinned buffer with a layout that depends
only on (tokens, sequences, block-table width), issues one ``cudaMemcpyAsync`` into a device buffer of
the same layout and runs the model on views of it. Decode steps replay a CUDA graph captured per
padded batch size (padding rows are real one-token sequences on the reserved block 0 / state slot 0,
so they never touch live memory), and speculative verify steps replay one captured per (padded batch
size, rows per sequence). Prefill steps run eagerly.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from ..models.hybrid import StepMeta
from .scheduler import SchedulerOutput

_FIELDS_T = ["input_ids", "positions", "slots", "tok_seq", "tok_ctx", "tok_state_slot", "tok_pos_in_chunk",
             "tok_has_state"]
_FIELDS_S = ["seq_state_slot", "seq_start", "seq_len", "seq_has_state"]


@dataclass
class Layout:
    T: int
    S: int
    MB: int
    R: int

    def offsets(self):
        off, o = {}, 0
        for f in _FIELDS_T:
            off[f] = o
            o += self.T
        for f in _FIELDS_S:
            off[f] = o
            o += self.S
        off["logits_idx"] = o
        o += self.R
        off["block_table"] = o
        o += self.S * self.MB
        return off, o


class MetaBuffers:
    def __init__(self, device, capacity: int):
        self.device = device
        self.capacity = capacity
        self.host = torch.zeros(capacity, dtype=torch.int32, pin_memory=True)
        self.dev = torch.zeros(capacity, dtype=torch.int32, device=device)
        self._views: dict[tuple, StepMeta] = {}

    def views(self, lay: Layout, write_state: bool = True) -> StepMeta:
        key = (lay.T, lay.S, lay.MB, lay.R, write_state)
        m = self._views.get(key)
        if m is None:
            off, total = lay.offsets()
            assert total <= self.capacity, "metadata buffer too small"
            d = self.dev
            kw = {f: d[off[f] : off[f] + lay.T] for f in _FIELDS_T}
            kw.update({f: d[off[f] : off[f] + lay.S] for f in _FIELDS_S})
            kw["logits_idx"] = d[off["logits_idx"] : off["logits_idx"] + lay.R]
            kw["block_table"] = d[off["block_table"] : off["block_table"] + lay.S * lay.MB].view(lay.S, lay.MB)
            m = StepMeta(write_state=write_state, **kw)
            self._views[key] = m
        return m


def _token_ids(seq, start: int, n: int) -> list[int]:
    """Tokens [start, start + n) of a sequence without joining its prompt and output."""
    P = len(seq.prompt)
    if start >= P:
        return seq.output[start - P : start - P + n]
    if start + n <= P:
        return seq.prompt[start : start + n]
    return seq.prompt[start:] + seq.output[: start + n - P]


def _block_row(seq) -> np.ndarray:
    """The sequence's block list as int32, rebuilt only when a block was added or the list replaced."""
    row = getattr(seq, "_bt_row", None)
    b = seq.blocks
    if row is None or row[0] is not b or row[1].shape[0] != len(b) or (b and row[1][-1] != b[-1]):
        row = (b, np.asarray(b, dtype=np.int32))
        seq._bt_row = row
    return row[1]


def pack_step(out: SchedulerOutput, block_size: int, pad_to_seqs: int = 0, draft: dict | None = None,
              pad_len: int = 1, mb: int | None = None):
    """Host-side metadata for a scheduled step: (Layout, np.int32 array). Sequences past the real ones
    (up to ``pad_to_seqs``) are padding of ``pad_len`` tokens each; every padding token is sampled.
    ``mb`` fixes the block-table width (a captured graph's); by default it is the widest sequence's."""
    chunks = out.chunks
    S_real = len(chunks)
    S = max(S_real, pad_to_seqs)
    toks, pos, slots, tseq, tctx, tslot, tpic, ths = [], [], [], [], [], [], [], []
    sslot, sstart, slen, shs = [], [], [], []
    logits_idx = []
    rows = [_block_row(ch.seq) for ch in chunks]
    MB = max([1] + [r.shape[0] for r in rows])
    if mb is not None:
        assert mb >= MB, "block table wider than the captured layout"
        MB = mb
    t = 0
    for i, ch in enumerate(chunks):
        seq = ch.seq
        ids = _token_ids(seq, ch.start, ch.n)
        d = draft.get(seq.seq_id) if draft is not None else None
        if d:
            ids = ids + d
        n = len(ids)
        blocks = seq.blocks
        hs = 1 if ch.start > 0 else 0
        toks.extend(ids)
        if n == 1:
            p0 = ch.start
            pos.append(p0)
            slots.append(blocks[p0 // block_size] * block_size + p0 % block_size)
            tctx.append(p0 + 1)
            tpic.append(0)
        else:
            p = np.arange(ch.start, ch.start + n, dtype=np.int64)
            pos.extend(p.tolist())
            slots.extend((rows[i][p // block_size].astype(np.int64) * block_size + p % block_size).tolist())
            tctx.extend((p + 1).tolist())
            tpic.extend(range(n))
        tseq.extend([i] * n)
        tslot.extend([seq.state_slot] * n)
        ths.extend([hs] * n)
        sslot.append(seq.state_slot)
        sstart.append(t)
        slen.append(n)
        shs.append(hs)
        if ch.sample:
            if d:
                logits_idx.extend(range(t + ch.n - 1, t + n))
            else:
                logits_idx.append(t + n - 1)
        t += n
    # padding sequences: pad_len tokens each on block 0 / state slot 0, no KV write
    for i in range(S_real, S):
        for j in range(pad_len):
            toks.append(0); pos.append(j); slots.append(-1); tseq.append(i); tctx.append(j + 1)
            tslot.append(0); tpic.append(j); ths.append(0)
            logits_idx.append(t + j)
        sslot.append(0); sstart.append(t); slen.append(pad_len); shs.append(0)
        t += pad_len
    T = t
    R = len(logits_idx)
    lay = Layout(T, S, MB, R)
    off, total = lay.offsets()
    arr = np.zeros(total, dtype=np.int32)
    for name, vals in (("input_ids", toks), ("positions", pos), ("slots", slots), ("tok_seq", tseq),
                       ("tok_ctx", tctx), ("tok_state_slot", tslot), ("tok_pos_in_chunk", tpic),
                       ("tok_has_state", ths), ("seq_state_slot", sslot), ("seq_start", sstart),
                       ("seq_len", slen), ("seq_has_state", shs), ("logits_idx", logits_idx)):
        arr[off[name] : off[name] + len(vals)] = vals
    bt = arr[off["block_table"] : off["block_table"] + S * MB].reshape(S, MB)
    for i, r in enumerate(rows):
        bt[i, : r.shape[0]] = r
    return lay, arr


class ModelRunner:
    def __init__(self, model, engine_cfg, block_size: int, max_tokens: int, max_seqs: int, max_blocks_per_seq: int):
        self.model = model
        from .. import knobs

        if knobs.get("R9K_TRACE") == "1" and getattr(model, "trace", None) is None:
            from ..utils.trace import DeviceTrace

            model.trace = DeviceTrace(model.device)
        self.cfg = engine_cfg
        self.device = model.device
        self.block_size = block_size
        self.max_blocks_per_seq = max_blocks_per_seq
        self.max_tokens = max_tokens
        self.max_seqs = max_seqs
        self.ws = model.alloc_workspace(max_tokens, max(max_seqs * (1 + engine_cfg.spec_tokens), max_seqs))
        cap = 8 * max_tokens + 5 * max_seqs + 2 * max_tokens + max_seqs * max_blocks_per_seq + 64
        self.meta = MetaBuffers(self.device, cap)
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.spec_graphs: dict[tuple[int, int], torch.cuda.CUDAGraph] = {}  # (batch, rows per sequence)
        self.graph_pool = None
        self.sample_out = torch.zeros(self.ws.logit_rows, dtype=torch.int64, device=self.device)
        self.sample_host = torch.zeros(self.ws.logit_rows, dtype=torch.int64, pin_memory=True)
        self.stream = torch.cuda.current_stream(self.device)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.device_events: list | None = None  # (start, end) CUDA events around each replayed step
        self.logit_log: list | None = None  # (seq_id, fp32 logits row on the host) per sampled row (tests)

    # ------------------------------------------------------------------------------------------
    def _upload(self, arr: np.ndarray) -> None:
        n = arr.size
        self.meta.host[:n].numpy()[:] = arr
        self.meta.dev[:n].copy_(self.meta.host[:n], non_blocking=True)
        self.h2d_bytes = n * 4

    def _graph_bs(self, S: int) -> int | None:
        if not self.cfg.cuda_graphs:
            return None
        for b in sorted(self.cfg.graph_batch_sizes):
            if b >= S and b in self.graphs:
                return b
        return None

    def capture_decode_graphs(self, max_blocks: int | None = None) -> None:
        """Capture one decode graph per batch size on padding-only batches."""
        from .scheduler import SchedulerOutput

        mb = max_blocks or self.max_blocks_per_seq
        for b in sorted(self.cfg.graph_batch_sizes):
            if b > self.max_seqs:
                continue
            lay, arr = pack_step(SchedulerOutput("decode", []), self.block_size, pad_to_seqs=b)
            lay = Layout(lay.T, lay.S, mb, lay.R)
            off, total = lay.offsets()
            arr2 = np.zeros(total, dtype=np.int32)
            small_off, _ = Layout(b, b, 1, b).offsets()
            for k in off:
                if k == "block_table":
                    continue
                ln = lay.T if k in _FIELDS_T else (lay.S if k in _FIELDS_S else lay.R)
                arr2[off[k] : off[k] + ln] = arr[small_off[k] : small_off[k] + ln]
            self._upload(arr2)
            meta = self.meta.views(lay)
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                for _ in range(2):
                    self.model.forward(meta, self.ws, lay.T, lay.R)
                    torch.argmax(self.ws.logits[: lay.R], dim=-1, out=self.sample_out[: lay.R])
            torch.cuda.current_stream(self.device).wait_stream(s)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.graph_pool):
                self.model.forward(meta, self.ws, lay.T, lay.R)
                torch.argmax(self.ws.logits[: lay.R], dim=-1, out=self.sample_out[: lay.R])
            self.graph_pool = g.pool()
            self.graphs[b] = g
        torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------------------------------------
    def execute(self, out: SchedulerOutput, sample: bool = True, draft=None, write_state: bool = True):
        """Run one scheduled step. Returns {seq_id: [token, ...]} (one token per sampled row)."""
        if not out.chunks:
            return {}
        gb = self._graph_bs(len(out.chunks)) if (out.kind == "decode" and draft is None) else None
        if gb is not None:
            lay, arr = pack_step(out, self.block_size, pad_to_seqs=gb, mb=self.max_blocks_per_seq)
            self._upload(arr)
            if self.device_events is not None:
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record()
                self.graphs[gb].replay()
                ev1.record()
                self.device_events.append((ev0, ev1))
            else:
                self.graphs[gb].replay()
            R = lay.R
        else:
            lay, arr = pack_step(out, self.block_size, draft=draft)
            self._upload(arr)
            meta = self.meta.views(lay, write_state=write_state)
            meta.host_seqs = _host_seqs(out, draft)
            meta.host_max_ctx = _host_max_ctx(out, draft)
            self.model.forward(meta, self.ws, lay.T, lay.R)
            R = lay.R
            torch.argmax(self.ws.logits[:R], dim=-1, out=self.sample_out[:R])
        if self.logit_log is not None:
            r = 0
            for ch in out.chunks:
                if ch.sample:
                    self.logit_log.append((ch.seq.seq_id, self.ws.logits[r].float().cpu()))
                    r += 1
        if not sample:
            return {}
        self.sample_host[:R].copy_(self.sample_out[:R], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        self.d2h_bytes = R * 8
        toks = self.sample_host[:R].tolist()
        res: dict[int, list[int]] = {}
        r = 0
        hot = []  # (logits row, params, generated so far) of rows that sample with temperature
        for ch in out.chunks:
            if not ch.sample:
                continue
            nd = len(draft[ch.seq.seq_id]) if draft is not None and ch.seq.seq_id in draft else 0
            res[ch.seq.seq_id] = toks[r : r + 1 + nd]
            if ch.seq.params.temperature > 0 and nd == 0:
                hot.append((r, ch.seq))
            r += 1 + nd
        if hot:
            self._resample(hot, res)
        return res

    def _resample(self, hot, res) -> None:
        from .sampler import sample_rows

        rows = torch.tensor([r for r, _ in hot], device=self.device)
        new = sample_rows(self.ws.logits.index_select(0, rows), [s.params for _, s in hot],
                          [len(s.output) for _, s in hot])
        for (_, s), t in zip(hot, new):
            res[s.seq_id] = [t]


    def _verify(self, meta: StepMeta, T: int, S: int) -> None:
        """Target forward over every verified row with the recurrent state read-only, the argmax of
        every row, greedy acceptance on the device and the commit of the accepted tokens."""
        from .. import _native

        self.model.forward(meta, self.ws, T, T)
        torch.argmax(self.ws.logits[:T], dim=-1, out=self.sample_out[:T])
        acc = self.ws.acc_len[:S]
        _native.ops().spec_accept(meta.input_ids, self.sample_out, meta.seq_start, meta.seq_len, acc)
        self.model.commit(meta, self.ws, acc)

    def _spec_graph(self, b: int, n: int) -> tuple[torch.cuda.CUDAGraph, Layout]:
        """The verify step of b sequences of n rows each (last token + n - 1 drafts) as a CUDA graph,
        captured on first use on a padding-only batch (block 0, state slot 0, no KV writes)."""
        from .scheduler import SchedulerOutput

        lay, arr = pack_step(SchedulerOutput("decode", []), self.block_size, pad_to_seqs=b, pad_len=n)
        lay_g = Layout(lay.T, lay.S, self.max_blocks_per_seq, lay.R)
        g = self.spec_graphs.get((b, n))
        if g is not None:
            return g, lay_g
        self._upload(_relayout(arr, lay, lay_g))
        meta = self.meta.views(lay_g, write_state=False)
        meta.host_seqs = [(i * n, n) for i in range(b)]  # every captured sequence has n rows
        meta.host_max_ctx = None
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._verify(meta, lay_g.T, b)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.graph_pool):
            self._verify(meta, lay_g.T, b)
        self.graph_pool = g.pool()
        self.spec_graphs[(b, n)] = g
        torch.cuda.synchronize(self.device)
        return g, lay_g

    def execute_spec(self, out: SchedulerOutput, draft: dict[int, list[int]]):
        """Speculative verify + commit: run [last token, drafts] of every sequence with the recurrent
        state read-only, take the target's argmax at every position, accept drafts greedily on the device,
        fold the accepted tokens into the GDN state (one launch) and return per sequence the accepted
        drafts plus the bonus token, and the number of verified positions committed. A step whose
        sequences all carry the same number of drafts replays a graph captured per (padded batch size,
        rows per sequence); other steps run eagerly."""
        n = _uniform_rows(out, draft)
        gb = self._graph_bs(len(out.chunks)) if n > 1 else None
        ev = None
        if self.device_events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        if gb is not None:
            g, lay_g = self._spec_graph(gb, n)
            lay, arr = pack_step(out, self.block_size, pad_to_seqs=gb, draft=draft, pad_len=n,
                                 mb=self.max_blocks_per_seq)
            self._upload(arr)
            if ev is not None:
                ev[0].record()
            g.replay()
        else:
            lay, arr = pack_step(out, self.block_size, draft=draft)
            assert lay.R == lay.T
            self._upload(arr)
            meta = self.meta.views(lay, write_state=False)
            meta.host_seqs = _host_seqs(out, draft)
            meta.host_max_ctx = _host_max_ctx(out, draft)
            if ev is not None:
                ev[0].record()
            self._verify(meta, lay.T, lay.S)
        if ev is not None:
            ev[1].record()
            self.device_events.append(ev)
        R = sum(1 + len(draft.get(ch.seq.seq_id, [])) for ch in out.chunks)  # real rows lead the padding
        self.sample_host[:R].copy_(self.sample_out[:R], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        self.d2h_bytes = R * 8
        y = self.sample_host[:R].tolist()
        res, accepted = {}, {}
        hot = []
        t = 0
        for ch in out.chunks:
            d = draft.get(ch.seq.seq_id, [])
            j = 0
            while j < len(d) and d[j] == y[t + j]:
                j += 1
            res[ch.seq.seq_id] = y[t: t + j + 1]
            accepted[ch.seq.seq_id] = j + 1
            if ch.seq.params.temperature > 0 and not d:
                hot.append((t, ch.seq))
            t += 1 + len(d)
        if hot:
            self._resample(hot, res)
        return res, accepted


def _uniform_rows(out: SchedulerOutput, draft: dict[int, list[int]]) -> int:
    """Rows per sequence when every sequence verifies one sampled token plus the same number of
    drafts (the shape a verify graph is captured for), else 0."""
    ns = {1 + len(draft.get(ch.seq.seq_id, [])) if ch.n == 1 and ch.sample else 0 for ch in out.chunks}
    return ns.pop() if len(ns) == 1 else 0


def _host_seqs(out: SchedulerOutput, draft=None) -> list[tuple[int, int]]:
    res, t = [], 0
    for ch in out.chunks:
        n = ch.n + (len(draft[ch.seq.seq_id]) if draft is not None and ch.seq.seq_id in draft else 0)
        res.append((t, n))
        t += n
    return res


def _host_max_ctx(out: SchedulerOutput, draft=None) -> int:
    """The longest attention context of any row of the step (position of its last token + 1)."""
    return max(ch.start + ch.n + (len(draft[ch.seq.seq_id]) if draft is not None and ch.seq.seq_id in draft else 0)
               for ch in out.chunks)


def _relayout(arr: np.ndarray, src: Layout, dst: Layout) -> np.ndarray:
    so, _ = src.offsets()
    do, total = dst.offsets()
    out = np.zeros(total, dtype=np.int32)
    for k in so:
        if k == "block_table":
            bt = arr[so[k] : so[k] + src.S * src.MB].reshape(src.S, src.MB)
            full = np.zeros((dst.S, dst.MB), dtype=np.int32)
            full[: src.S, : src.MB] = bt
            out[do[k] : do[k] + dst.S * dst.MB] = full.reshape(-1)
        else:
            ln = src.T if k in _FIELDS_T else (src.S if k in _FIELDS_S else src.R)
            out[do[k] : do[k] + ln] = arr[so[k] : so[k] + ln]
    return out
