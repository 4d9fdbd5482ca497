"""Host-side speculative decoding logic: drafters' proposals, adaptive k, scheduler accounting."""
from r9700_stack_b200.engine.scheduler import SamplingParams, ScheduledChunk, Scheduler, SchedulerOutput, Sequence
from r9700_stack_b200.spec.drafters import AdaptiveK, NgramDrafter, ScriptedDrafter


def test_ngram_prompt_lookup():
    d = NgramDrafter(3)
    s = Sequence([1, 2, 3, 4, 5, 9, 2, 3], SamplingParams())
    # last tokens "2 3" occurred at 1..2, followed by 4 5 9
    assert d.propose_host(s) == [4, 5, 9]
    s2 = Sequence([7, 8], SamplingParams())
    assert d.propose_host(s2) == [8, 8, 8]  # no match: repeat the last token
    s3 = Sequence([1, 2, 1], SamplingParams())
    assert d.propose_host(s3) == [2, 1, 1]  # short continuation padded


def test_scripted_drafter_positions():
    s = Sequence([1], SamplingParams())
    d = ScriptedDrafter(3, {s.seq_id: [10, 11, 12, 13, 14]}, pad=0)
    assert d.drafts([s]) == {s.seq_id: [10, 11, 12]}
    s.output = [10, 11]
    assert d.drafts([s]) == {s.seq_id: [12, 13, 14]}
    s.output = [10, 11, 12, 13]
    assert d.drafts([s]) == {s.seq_id: [14, 0, 0]}


def test_adaptive_k():
    a = AdaptiveK(5, 1)
    assert a.update(5, 0) == 4
    assert a.update(4, 1) == 3
    assert a.update(3, 3) == 4
    for _ in range(5):
        a.update(5, 5)
    assert a.k == 5


def test_scheduler_spec_accounting():
    sch = Scheduler(num_blocks=64, num_slots=4, block_size=4, max_batch=2, max_prefill_tokens=64, max_model_len=128)
    seq = Sequence(list(range(10)), SamplingParams(max_tokens=20))
    sch.add(seq)
    out = sch.schedule(lookahead=4)
    assert out.kind == "prefill"
    sch.finish_step(out, {seq.seq_id: [42]})
    assert seq.num_computed == 10 and seq.length == 11
    out = sch.schedule(lookahead=4)
    assert out.kind == "decode" and out.chunks[0].start == 10
    # blocks cover the verify positions 10..13
    assert len(seq.blocks) * 4 >= 14
    # verify accepted 2 drafts + bonus -> 3 new tokens, 13 cached
    sch.finish_step(out, {seq.seq_id: [1, 2, 3]})
    assert seq.length == 14 and seq.num_computed == 13
    assert sch.ensure(seq, 30) and len(seq.blocks) * 4 >= 30
