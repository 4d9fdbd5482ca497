"""Draft proposers for speculative decoding.

A drafter keeps, per running sequence, the k tokens it proposes for the next verify step. The engine
calls :meth:`Drafter.after_step` once a target step (prefill chunk, decode or verify) has been
committed, with the target's final residual rows still in the runner's workspace; the drafter
updates its own context from them and prepares the next proposal.

* :class:`NgramDrafter` - prompt lookup (host only): the continuation after the latest earlier
  occurrence of the sequence's last n tokens.
* :class:`ScriptedDrafter` - proposes a given continuation (tests, replays).
* :class:`ModelDrafter` - the one-layer MTP head (k sequential drafts, shared weights) or the
  DFlash-style block drafter (k drafts in one forward) of :mod:`.draft_model`.

Reference: r9700_vllm/spec/mtp_rocm.py:21-57, r9700_vllm/models/dflash.py:26-230, and the DSpark
drafter with adaptive verification (r9700_vllm/dsv4_glue.py:812), whose confidence-based draft
length is :class:`AdaptiveK`.
"""
from __future__ import annotations

import numpy as np
import torch

from ..engine.runner import Layout, MetaBuffers
from ..engine.scheduler import Sequence, SchedulerOutput


class Drafter:
    def __init__(self, k: int):
        self.k = k
        self.pending: dict[int, list[int]] = {}

    def drafts(self, seqs: list[Sequence]) -> dict[int, list[int]]:
        """Proposals for the given sequences (up to k tokens each; sequences without one get none)."""
        out = {}
        for s in seqs:
            d = self.pending.get(s.seq_id)
            if d is None:
                d = self.propose_host(s)
            if d:
                out[s.seq_id] = list(d[: self.k])
        return out

    def propose_host(self, seq: Sequence) -> list[int] | None:
        return None

    def after_step(self, engine, out: SchedulerOutput, accepted: dict[int, int] | None,
                   drafts: dict[int, list[int]] | None) -> None:
        pass

    def release(self, seq: Sequence) -> None:
        self.pending.pop(seq.seq_id, None)


class NgramDrafter(Drafter):
    """Prompt-lookup decoding: match the last n (n_max..n_min) tokens earlier in the sequence and
    propose what followed; pads with the last token when nothing matches."""

    def __init__(self, k: int, n_max: int = 4, n_min: int = 1):
        super().__init__(k)
        self.n_max, self.n_min = n_max, n_min

    def propose_host(self, seq: Sequence) -> list[int]:
        toks = seq.tokens
        L = len(toks)
        arr = np.asarray(toks, dtype=np.int64)
        for n in range(min(self.n_max, L - 1), self.n_min - 1, -1):
            pat = arr[L - n:]
            # latest earlier occurrence whose continuation exists
            for st in range(L - n - 1, -1, -1):
                if np.array_equal(arr[st:st + n], pat):
                    cont = toks[st + n: st + n + self.k]
                    if cont:
                        return (cont + [cont[-1]] * self.k)[: self.k]
        return [toks[-1]] * self.k


class ScriptedDrafter(Drafter):
    """Proposes script[seq_id][len(output):len(output)+k] (a known continuation), padded with
    ``pad``; ``corrupt_every`` replaces every n-th proposal with ``pad`` to exercise rejection."""

    def __init__(self, k: int, script: dict[int, list[int]], pad: int = 0, corrupt_every: int = 0):
        super().__init__(k)
        self.script, self.pad, self.corrupt_every = script, pad, corrupt_every
        self._n = 0

    def propose_host(self, seq: Sequence) -> list[int]:
        cont = self.script.get(seq.seq_id, [])[len(seq.output): len(seq.output) + self.k]
        cont = cont + [self.pad] * (self.k - len(cont))
        if self.corrupt_every:
            for i in range(self.k):
                self._n += 1
                if self._n % self.corrupt_every == 0:
                    cont[i] = self.pad
        return cont


class AdaptiveK:
    """Adaptive verification length: shrink k after rejections, grow it after full acceptance
    (the DSpark policy's role), within [k_min, k_max]."""

    def __init__(self, k_max: int, k_min: int = 1):
        self.k_max, self.k_min = k_max, k_min
        self.k = k_max

    def update(self, n_drafted: int, n_accepted: int) -> int:
        if n_accepted >= n_drafted:
            self.k = min(self.k_max, self.k + 1)
        elif n_accepted < n_drafted // 2:
            self.k = max(self.k_min, self.k - 1)
        return self.k


def _slots(seq: Sequence, pos: np.ndarray, bs: int) -> np.ndarray:
    b = np.asarray(seq.blocks, dtype=np.int64)
    return b[pos // bs] * bs + pos % bs


class ModelDrafter(Drafter):
    """GPU drafter: MTP head (``kind="mtp"``) or block drafter (``kind="block"``)."""

    def __init__(self, target_model, kind: str, k: int, engine_cfg, num_blocks: int, num_slots: int,
                 seed: int = 0):
        from .draft_model import build_draft_model

        super().__init__(k)
        assert kind in ("mtp", "block")
        self.kind = kind
        self.model = build_draft_model(target_model, kind, seed=seed)
        self.bs = engine_cfg.kv_block
        self.model.alloc_caches(num_blocks, num_slots, engine_cfg.kv_block)
        mb = engine_cfg.max_batch
        self.max_tokens = engine_cfg.max_prefill_tokens + mb * (k + 2)
        self.ws = self.model.alloc_workspace(self.max_tokens, max(mb * (k + 1), mb))
        dev = self.model.device
        self.meta = MetaBuffers(dev, 8 * self.max_tokens + 8 * mb + mb * 4096 + 64)
        self.h_idx = torch.zeros(self.max_tokens, dtype=torch.int32, device=dev)
        self.row_kind = torch.zeros(self.max_tokens, dtype=torch.int32, device=dev)
        self._h_host = torch.zeros(2 * self.max_tokens, dtype=torch.int32, pin_memory=True)
        self.model.h_idx, self.model.row_kind = self.h_idx, self.row_kind
        self.sample = torch.zeros(self.ws.logit_rows, dtype=torch.int64, device=dev)

    # ------------------------------------------------------------------------------------------
    def _run(self, groups, h_src: torch.Tensor) -> list[int]:
        """groups: per sequence (seq, tokens, positions, ctx, h_rows, kinds, logit_rows_local).
        Runs one drafter forward; returns the argmax token of every requested logits row."""
        toks, pos, slots, tseq, tctx, hrow, kinds, lidx = [], [], [], [], [], [], [], []
        sstart, slen = [], []
        MB = max(len(g[0].blocks) for g in groups)
        bt = np.zeros((len(groups), MB), dtype=np.int32)
        t = 0
        for i, (seq, tk, ps, cx, hr, kd, lr) in enumerate(groups):
            n = len(tk)
            toks += tk; pos += ps; tctx += cx; hrow += hr; kinds += kd
            slots += _slots(seq, np.asarray(ps, dtype=np.int64), self.bs).tolist()
            tseq += [i] * n
            sstart.append(t); slen.append(n)
            lidx += [t + r for r in lr]
            bt[i, : len(seq.blocks)] = seq.blocks
            t += n
        T, S, R = t, len(groups), len(lidx)
        lay = Layout(T, S, MB, R)
        off, total = lay.offsets()
        arr = np.zeros(total, dtype=np.int32)
        z = [0] * T
        for name, vals in (("input_ids", toks), ("positions", pos), ("slots", slots), ("tok_seq", tseq),
                           ("tok_ctx", tctx), ("tok_state_slot", z), ("tok_pos_in_chunk", z),
                           ("tok_has_state", z), ("seq_state_slot", [0] * S), ("seq_start", sstart),
                           ("seq_len", slen), ("seq_has_state", [0] * S), ("logits_idx", lidx)):
            arr[off[name]: off[name] + len(vals)] = vals
        arr[off["block_table"]: off["block_table"] + S * MB] = bt.reshape(-1)
        self.meta.host[:total].numpy()[:] = arr
        self.meta.dev[:total].copy_(self.meta.host[:total], non_blocking=True)
        hh = self._h_host.numpy()
        hh[:T] = hrow
        hh[T:2 * T] = kinds
        self.h_idx[:T].copy_(self._h_host[:T], non_blocking=True)
        self.row_kind[:T].copy_(self._h_host[T:2 * T], non_blocking=True)
        meta = self.meta.views(lay)
        meta.host_seqs = list(zip(sstart, slen))
        self.model.h_src = h_src
        self.model.forward(meta, self.ws, T, R)
        torch.argmax(self.ws.logits[:R], dim=-1, out=self.sample[:R])
        return self.sample[:R].tolist()

    def after_step(self, engine, out: SchedulerOutput, accepted, drafts) -> None:
        """Feed the target positions this step committed and propose the next drafts."""
        runner, sched = engine.runner, engine.scheduler
        h_tgt = runner.ws.resid
        feed = []  # (seq, positions, target rows, propose?)
        t = 0
        for ch in out.chunks:
            seq = ch.seq
            nd = len(drafts.get(seq.seq_id, [])) if drafts else 0
            n_rows = ch.n + nd
            if out.kind == "prefill":
                npos = ch.n
            else:
                npos = accepted.get(seq.seq_id, 1) if accepted else 1
            if not seq.finished:
                ps = list(range(ch.start, ch.start + npos))
                feed.append((seq, ps, [t + i for i in range(npos)], ch.sample))
            t += n_rows
        for f in feed:
            self.pending.pop(f[0].seq_id, None)
        if not feed:
            return
        if self.kind == "mtp":
            self._mtp(feed, h_tgt, sched)
        else:
            self._block(feed, h_tgt, sched)

    def _mtp(self, feed, h_tgt, sched) -> None:
        groups, props = [], []
        for seq, ps, rows, propose in feed:
            toks = seq.tokens
            # pair (h_p, x_{p+1}) at position p; x_{p+1} always exists once the step is committed
            ok = [i for i, p in enumerate(ps) if p + 1 < len(toks)]
            if not ok:
                continue
            ps2 = [ps[i] for i in ok]
            propose = propose and ps2[-1] + 1 == len(toks) - 1 and sched.ensure(seq, ps2[-1] + self.k + 1)
            groups.append((seq, [toks[p + 1] for p in ps2], ps2, [p + 1 for p in ps2], [rows[i] for i in ok],
                           [0] * len(ps2), [len(ps2) - 1] if propose else []))
            props.append(propose)
        if not groups:
            return
        first = self._run(groups, h_tgt)
        live = [(g[0], g[2][-1]) for g, p in zip(groups, props) if p]
        cur = {s.seq_id: [d] for (s, _), d in zip(live, first)}
        for m in range(1, self.k):
            gs = []
            for j, (s, plast) in enumerate(live):
                p = plast + m
                gs.append((s, [cur[s.seq_id][-1]], [p], [p + 1], [j], [0], [0]))
            nxt = self._run(gs, self.ws.h_out)
            for (s, _), d in zip(live, nxt):
                cur[s.seq_id].append(d)
        self.pending.update(cur)

    def _block(self, feed, h_tgt, sched) -> None:
        B = self.k + 1
        groups = []
        for seq, ps, rows, propose in feed:
            L = seq.length
            tk = [0] * len(ps)
            cx = [p + 1 for p in ps]
            kd = [-1] * len(ps)
            hr = list(rows)
            lr = []
            pos = list(ps)
            if propose and sched.ensure(seq, L - 1 + B):
                q0 = L - 1
                pos += list(range(q0, q0 + B))
                tk += [seq.tokens[-1]] + [0] * (B - 1)
                cx += [q0 + B] * B
                kd += [0] + [1] * (B - 1)
                hr += [0] * B
                lr = list(range(len(ps) + 1, len(ps) + B))
            groups.append((seq, tk, pos, cx, hr, kd, lr))
        res = self._run(groups, h_tgt)
        i = 0
        for g in groups:
            n = len(g[6])
            if n:
                self.pending[g[0].seq_id] = res[i:i + n]
            i += n


class DSparkDrafter(ModelDrafter):
    """DSpark-style drafter: the block drafter's per-position logits refined left to right by a
    low-rank Markov head conditioned on the previous draft token, plus a confidence head that cuts
    each sequence's draft where the running confidence drops below ``min_conf`` (adaptive
    verification length per sequence; at least one draft is kept).

      logits_j = block_logits_j + W_head @ E_markov[d_{j-1}]       (rank-r bigram correction)
      conf_j   = sigmoid(w_conf . [h_j, E_markov[d_j]])             (h_j: drafter output row)

    Reference: r9700_vllm/dsv4_glue.py:812 (install_markov), kernels/r9k_dsv4_glue.hip:500-649
    (r9k_dsv4_markov_kernel / _last / _conf), the pack's mtp.0.markov_head / confidence_head tensors.
    """

    def __init__(self, target_model, k: int, engine_cfg, num_blocks: int, num_slots: int, seed: int = 0,
                 rank: int = 64, min_conf: float = 0.3):
        super().__init__(target_model, "block", k, engine_cfg, num_blocks, num_slots, seed=seed)
        from ..models.weights import WeightFactory
        from ..ops import linear as L

        c, dev = self.model.cfg, self.model.device
        wf = WeightFactory(dev, seed=seed * 1000 + 4242, std=0.02)
        V = self.model.vocab_local * self.model.par.tp_size
        self.markov_embed = wf.randn(V, rank, dtype=torch.bfloat16)
        self.markov_head = L.BF16Weight(wf.randn(V, rank, dtype=torch.bfloat16))
        self.conf_w = L.BF16Weight(wf.randn(1, c.hidden + rank, std=0.05, dtype=torch.bfloat16))
        self.min_conf = min_conf
        self.vocab = V
        mb, km, grid = engine_cfg.max_batch, k, -(-V // 512)
        # refinement state on the device: drafts, running confidence, kept lengths, the per-CTA
        # maxima of one launch and its arrival counter (re-armed by the launch itself)
        self._mk_state = (torch.zeros(mb * km, dtype=torch.int64, device=dev),
                          torch.zeros(mb, dtype=torch.float32, device=dev),
                          torch.zeros(mb, dtype=torch.int32, device=dev),
                          torch.zeros(64 * grid * 2, dtype=torch.float32, device=dev),
                          torch.zeros(1, dtype=torch.int32, device=dev))
        self.last_lengths: list[int] = []

    def _block(self, feed, h_tgt, sched) -> None:
        super()._block(feed, h_tgt, sched)  # fills self.ws.logits rows (B-1 per proposing sequence)
        prop = [f[0] for f in feed if f[0].seq_id in self.pending]
        if not prop:
            return
        S, km, V = len(prop), self.k, self.vocab
        base = self.ws.logits[: S * km].view(S, km, V)
        hrows = self.ws.h_out[: S * km].view(S, km, -1)
        prev = torch.tensor([s.tokens[-1] for s in prop], dtype=torch.int64, device=self.model.device)
        dl, ln = self.refine(base, hrows, prev)
        self.last_lengths = ln
        for s, row, n in zip(prop, dl, ln):
            self.pending[s.seq_id] = row[: max(1, n)]

    def refine(self, base: torch.Tensor, hrows: torch.Tensor, prev: torch.Tensor):
        """Markov-refined drafts [S][k] and kept lengths [S] from the block drafter's logits
        base [S, k, V] (fp32), its output rows hrows [S, k, H] and the last target token of every
        sequence: one ``dspark_markov_step`` launch per draft position, one copy to the host."""
        from .. import _native

        S, km, V = base.shape
        drafts, run, lengths, part, counter = self._mk_state
        assert S * km <= drafts.numel(), "more proposing sequences than the engine's batch"
        base, hrows, prev = base.contiguous(), hrows.contiguous(), prev.clone()
        w_conf = self.conf_w.w.reshape(-1)
        ops = _native.ops()
        for c0 in range(0, S, 64):  # the kernel holds up to 64 sequences' embeddings in shared memory
            c1 = min(S, c0 + 64)
            for j in range(km):
                ops.dspark_markov_step(base[c0:c1], j, self.markov_embed, self.markov_head.w, hrows[c0:c1], w_conf,
                                       float(self.min_conf), prev[c0:c1], run[c0:c1], lengths[c0:c1],
                                       drafts[c0 * km:c1 * km], part, counter)
        host = torch.cat([drafts[: S * km], lengths[:S].long()]).cpu()
        return host[: S * km].view(S, km).tolist(), host[S * km:].tolist()

    def refine_reference(self, base: torch.Tensor, hrows: torch.Tensor, prev: torch.Tensor):
        """The same refinement as :meth:`refine` in plain torch ops (fp32 logits), for tests."""
        from ..ops import linear as L

        S, km, V = base.shape
        dev = base.device
        drafts, conf_run = [], torch.ones(S, device=dev)
        keep = torch.ones(S, dtype=torch.bool, device=dev)
        lengths = torch.zeros(S, dtype=torch.int64, device=dev)
        H = hrows.shape[-1]
        mk = torch.zeros(S, V, dtype=torch.float32, device=dev)
        cat = torch.zeros(S, H + self.markov_embed.shape[1], dtype=torch.bfloat16, device=dev)
        conf = torch.zeros(S, 1, dtype=torch.float32, device=dev)
        for j in range(km):
            e_prev = self.markov_embed.index_select(0, prev)
            L.bf16_linear(e_prev, self.markov_head, out=mk, out_dtype=torch.float32)
            d = torch.argmax(base[:, j] + mk, dim=-1)
            cat[:, :H].copy_(hrows[:, j])
            cat[:, H:].copy_(self.markov_embed.index_select(0, d))
            L.bf16_linear(cat, self.conf_w, out=conf, out_dtype=torch.float32)
            conf_run = conf_run * torch.sigmoid(conf[:, 0])
            keep = keep & ((conf_run >= self.min_conf) | (j == 0))
            lengths += keep.long()
            drafts.append(d)
            prev = d
        return torch.stack(drafts, 1).tolist(), lengths.tolist()
