"""Scheduler, allocators and step-metadata packing (host-only logic)."""
import numpy as np
import pytest

from r9700_stack_b200.engine.cache import BlockAllocator
from r9700_stack_b200.engine.runner import Layout, pack_step, _relayout
from r9700_stack_b200.engine.scheduler import SamplingParams, Scheduler, Sequence


def test_block_allocator_order_and_errors():
    a = BlockAllocator(5)
    assert a.allocate(2) == [1, 2]
    a.free([1])
    assert a.allocate(1) == [1]
    with pytest.raises(MemoryError):
        a.allocate(10)
    with pytest.raises(ValueError):
        a.free([0])


def _sched(**kw):
    d = dict(num_blocks=64, num_slots=5, block_size=4, max_batch=4, max_prefill_tokens=16, max_model_len=256)
    d.update(kw)
    return Scheduler(**d)


def test_chunked_prefill_then_decode():
    s = _sched()
    seq = Sequence(list(range(20)), SamplingParams(max_tokens=3))
    s.add(seq)
    o1 = s.schedule()
    assert o1.kind == "prefill" and o1.chunks[0].n == 16 and not o1.chunks[0].sample
    s.finish_step(o1, {})
    o2 = s.schedule()
    assert o2.kind == "prefill" and o2.chunks[0].start == 16 and o2.chunks[0].n == 4 and o2.chunks[0].sample
    s.finish_step(o2, {seq.seq_id: [7]})
    assert seq.output == [7] and seq.num_computed == 20
    o3 = s.schedule()
    assert o3.kind == "decode" and o3.chunks[0].start == 20
    s.finish_step(o3, {seq.seq_id: [8]})
    o4 = s.schedule()
    s.finish_step(o4, {seq.seq_id: [9]})
    assert seq.finished and seq.output == [7, 8, 9]
    assert s.blocks.num_free == 63 and s.slots.num_free == 4


def test_pack_step_metadata():
    s = _sched()
    a = Sequence(list(range(6)), SamplingParams(max_tokens=2))
    b = Sequence(list(range(3)), SamplingParams(max_tokens=2))
    s.add(a); s.add(b)
    out = s.schedule()
    lay, arr = pack_step(out, 4, pad_to_seqs=3)
    off, total = lay.offsets()
    assert lay.T == 10 and lay.S == 3 and lay.R == 3
    pos = arr[off["positions"]:off["positions"] + lay.T]
    assert pos.tolist() == [0, 1, 2, 3, 4, 5, 0, 1, 2, 0]
    slots = arr[off["slots"]:off["slots"] + lay.T]
    assert slots[-1] == -1  # padding row writes no KV
    bt = arr[off["block_table"]:off["block_table"] + lay.S * lay.MB].reshape(lay.S, lay.MB)
    assert slots[4] == bt[0, 1] * 4 + 0
    li = arr[off["logits_idx"]:off["logits_idx"] + lay.R]
    assert li.tolist() == [5, 8, 9]
    big = Layout(lay.T, lay.S, 7, lay.R)
    arr2 = _relayout(arr, lay, big)
    off2, _ = big.offsets()
    bt2 = arr2[off2["block_table"]:off2["block_table"] + big.S * big.MB].reshape(big.S, big.MB)
    assert (bt2[:, :lay.MB] == bt).all() and (bt2[:, lay.MB:] == 0).all()


def test_pack_step_decode_fast_path_matches_relayout():
    """Decode packing (one token per sequence, read without joining prompt and output, block rows
    cached per sequence) written straight at a graph's table width equals the default packing
    re-laid to that width; drafts extend a row; a chunk straddling prompt and output reads both."""
    s = _sched()
    a = Sequence(list(range(6)), SamplingParams(max_tokens=8))
    b = Sequence(list(range(3)), SamplingParams(max_tokens=8))
    s.add(a); s.add(b)
    s.finish_step(s.schedule(), {a.seq_id: [40], b.seq_id: [50]})
    for step in range(3):
        out = s.schedule()
        lay, arr = pack_step(out, 4, pad_to_seqs=4)
        lay_w, arr_w = pack_step(out, 4, pad_to_seqs=4, mb=9)
        assert (lay_w.T, lay_w.S, lay_w.MB, lay_w.R) == (lay.T, lay.S, 9, lay.R)
        assert (arr_w == _relayout(arr, lay, Layout(lay.T, lay.S, 9, lay.R))).all()
        off, _ = lay.offsets()
        assert arr[off["input_ids"]:off["input_ids"] + 2].tolist() == [a.tokens[-1], b.tokens[-1]]
        s.finish_step(out, {a.seq_id: [41 + step], b.seq_id: [51 + step]})
    out = s.schedule(lookahead=3)
    lay, arr = pack_step(out, 4, draft={a.seq_id: [7, 8]})
    off, _ = lay.offsets()
    assert arr[off["input_ids"]:off["input_ids"] + lay.T].tolist() == [a.tokens[-1], 7, 8, b.tokens[-1]]
    assert arr[off["positions"]:off["positions"] + 3].tolist() == [a.length - 1, a.length, a.length + 1]
    from r9700_stack_b200.engine.runner import _token_ids

    assert _token_ids(a, 4, 4) == a.tokens[4:8]


def test_preemption_when_out_of_blocks():
    s = _sched(num_blocks=6, block_size=4, max_prefill_tokens=64)
    seqs = [Sequence(list(range(7)), SamplingParams(max_tokens=8)) for _ in range(2)]
    for q in seqs:
        s.add(q)
    out = s.schedule()
    s.finish_step(out, {q.seq_id: [1] for q in seqs})
    for _ in range(4):
        out = s.schedule()
        s.finish_step(out, {c.seq.seq_id: [1] for c in out.chunks if c.sample})
    assert len(s.running) + len(s.waiting) + len(s.finished) == 2
