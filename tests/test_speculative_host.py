"""The self-speculative decoder's control flow on CPU (speculative.js:58-189):
drafting with the first layers, token-by-token verification, rollback to the
first mismatch, the bonus token and EOS handling.  A deterministic stand-in
runtime gives each step's greedy token: the full model maps token t to
f(t); the draft agrees except on tokens divisible by 3.  Greedy speculative
output must equal plain greedy decoding of the full model."""
import pytest

from purebee_b200.speculative import SelfSpeculativeDecoder

V = 101


def full_next(t):
    return (7 * t + 3) % V


def draft_next(t):
    return full_next(t) if t % 3 else (full_next(t) + 1) % V


class StandInRuntime:
    n_layers = 8

    def __init__(self):
        self.calls = []

    def resetCache(self):
        self.calls.append(("reset",))

    def rollbackCache(self, pos):
        self.calls.append(("rollback", pos))

    def forward(self, tokens, start):
        logits = [0.0] * V
        logits[full_next(tokens[-1])] = 1.0
        return {"logits": logits}

    def argmax(self, logits):
        return max(range(len(logits)), key=lambda i: (logits[i], -i))

    def step(self, token, pos, max_layers=0):
        self.calls.append(("step", token, pos, max_layers))
        return draft_next(token) if max_layers else full_next(token)


def greedy_chain(last, n, eos=()):
    out = []
    t = last
    for _ in range(n):
        t = full_next(t)
        out.append(t)
        if t in eos:
            break
    return out


@pytest.mark.parametrize("draft_count", [1, 3, 4, 6])
def test_greedy_output_equals_full_model(draft_count):
    rt = StandInRuntime()
    dec = SelfSpeculativeDecoder(rt, {"draftLayers": 2, "draftCount": draft_count})
    prompt = [5, 9, 12]
    res = dec.generate(prompt, 40, {"greedy": True, "eosIds": [-1]})
    assert res["tokens"][:3] == prompt
    assert res["tokens"][3:] == greedy_chain(prompt[-1], len(res["tokens"]) - 3)
    assert res["generated"] == len(res["tokens"]) - 3 and 40 <= res["generated"] <= 40 + draft_count
    st = dec.stats
    assert 0 < st["totalAccepted"] < st["totalDrafted"]  # the draft disagrees on some tokens
    # drafts run with the layer limit, verification with the full model
    assert {c[3] for c in rt.calls if c[0] == "step"} == {0, 2}


def test_stops_at_eos():
    rt = StandInRuntime()
    dec = SelfSpeculativeDecoder(rt, {"draftLayers": 2, "draftCount": 4})
    prompt = [5]
    chain = greedy_chain(prompt[-1], 30)
    eos = chain[11]
    res = dec.generate(prompt, 30, {"greedy": True, "eosIds": [eos]})
    assert res["tokens"][1:] == greedy_chain(prompt[-1], 30, eos=(eos,))
    assert res["tokens"][-1] == eos


def test_rollback_positions_stay_in_range():
    rt = StandInRuntime()
    dec = SelfSpeculativeDecoder(rt, {"draftLayers": 3, "draftCount": 4})
    prompt = [1, 2, 3, 4]
    res = dec.generate(prompt, 25, {"greedy": True, "eosIds": [-1]})
    end = len(res["tokens"])
    for c in rt.calls:
        if c[0] == "rollback":
            assert len(prompt) <= c[1] <= end
        if c[0] == "step":
            assert len(prompt) <= c[2] < end
