"""Accuracy gates on CPU with stand-in engines: McNemar's exact test, answer scoring in GSM8K's
format, the paired comparison and selftest, needle prompts, and the drafter self-test verdicts."""
import math

from r9700_stack_b200.serve import evals as E
from r9700_stack_b200.serve.tokenizer import ByteTokenizer


def test_mcnemar_exact():
    assert E.mcnemar_exact(0, 0) == 1.0
    # 10 discordant pairs all one way: 2 * 0.5^10
    assert math.isclose(E.mcnemar_exact(10, 0), 2 * 0.5 ** 10)
    assert E.mcnemar_exact(5, 5) == 1.0
    assert E.mcnemar_exact(3, 12) < 0.05 < E.mcnemar_exact(5, 9)


def test_scoring():
    it = {"question": "q", "answer": "so 1,234 + 1 = 1,235 #### 1,235"}
    assert E.reference_answer(it) == "1235"
    assert E.score("The answer is 1235.", it) and E.score("... 1,235", it)
    assert not E.score("12", it) and not E.score("no number", it)


class _Oracle:
    """Answers arith items correctly except those whose index is in `wrong`."""

    def __init__(self, items, wrong=()):
        self.tok, self.items, self.wrong = ByteTokenizer(), items, set(wrong)

    def generate(self, prompts, params):
        out = []
        for p in prompts:
            q = self.tok.decode(p)
            i = next(k for k, it in enumerate(self.items) if it["question"] in q)
            ans = E.reference_answer(self.items[i])
            out.append(self.tok.encode(" 0" if i in self.wrong else f" {ans}"))
        return out


def test_paired_and_selftest():
    items = E.arith_task(60, seed=3)
    tok = ByteTokenizer()
    same = E.paired(_Oracle(items), _Oracle(items), tok, items)
    assert same["b_base_only"] == same["c_cand_only"] == 0 and same["pass"]
    worse = E.paired(_Oracle(items), _Oracle(items, wrong=range(0, 40, 2)), tok, items)
    assert worse["b_base_only"] == 20 and worse["different"] and not worse["pass"]
    better = E.paired(_Oracle(items, wrong=range(20)), _Oracle(items), tok, items)
    assert better["different"] and better["pass"]  # a significant gain is not a failure
    st = E.selftest(_Oracle(items), tok, items)
    assert st["text_disagreement"] == 0.0 and st["pass"]


def test_needle_prompt_layout():
    key, value = [10, 11, 12, 13], [20, 21, 22, 23]
    p = E.needle_prompt(100, 0.5, key, value, vocab=512, seed=1)
    assert len(p) == 100 and p[-4:] == key
    i = p.index(10)
    assert p[i:i + 8] == key + value


class _Echo:
    def __init__(self, answer):
        self.answer = answer
        self.spec_stats = {"drafted": 10, "accepted": 7}

    def generate(self, prompts, params):
        return [self.answer(p) for p in prompts]


def test_drafter_selftest_verdicts():
    ps = [[1, 2, 3], [4, 5]]
    ok = E.drafter_selftest(_Echo(lambda p: p[::-1]), _Echo(lambda p: p[::-1]), ps)
    assert ok["pass"] and ok["acceptance"] == 0.7
    bad = E.drafter_selftest(_Echo(lambda p: p[::-1]), _Echo(lambda p: p), ps)
    assert not bad["pass"] and bad["mismatched"] == [0, 1]


def test_needles_harness():
    key_value = {}

    class _Recall:
        def generate(self, prompts, params):
            p = prompts[0]
            k = p[-4:]
            for i in range(len(p) - 8):
                if p[i:i + 4] == k:
                    return [p[i + 4:i + 8]]
            return [[0, 0, 0, 0]]

    r = E.needles(_Recall(), 256, [0.1, 0.5, 0.9], vocab=512, trials=2)
    assert r["pass"] and r["found"] == 6
