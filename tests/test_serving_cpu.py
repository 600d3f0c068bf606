"""The continuous-batching scheduler (serving.Server) on the CPU, over a stand-in execution
whose next token depends only on the request's seed, its draw index and its prompt -- the
property the real engine has (each request draws from its own Rng, whatever else is in the
batch). Checked: every request's tokens equal the same request served alone; requests end
after emitting the end-of-sequence token ("stop") or at their token budget ("length");
no more slots are busy than exist and freed slots are refilled from the queue; every slot
is released once per request; prompts that do not fit the context are refused."""
import numpy as np
import pytest

from cpp_inference_train_engine_b200.config import ModelConfig
from cpp_inference_train_engine_b200.engine import EngineError
from cpp_inference_train_engine_b200.serving import Server

V = 64
EOS = V - 6


def _token(seed, draw, prompt_sum):
    x = (int(seed) * 0x9E3779B1 + int(draw) * 0x85EBCA77 + int(prompt_sum) * 0xC2B2AE3D) & 0xFFFFFFFF
    x ^= x >> 15
    return int(x % V)


class FakeExecution:
    """serve_open / serve_admit / serve_step / serve_release with per-request tokens."""

    def __init__(self):
        self.cfg = ModelConfig(vocab_size=V, max_sequence_length=64)
        self.slots = None
        self.busy = []
        self.prompt_sum = {}
        self.max_busy = 0
        self.released = []

    def serve_open(self, slots, max_context):
        self.slots = slots
        self.max_context = max_context
        self.busy = [False] * slots

    def serve_admit(self, slot, prompt, max_new, temperature, seed):
        assert not self.busy[slot], "admitted into a busy slot"
        assert prompt.size + max_new <= self.max_context
        self.busy[slot] = True
        self.max_busy = max(self.max_busy, sum(self.busy))
        self.prompt_sum[slot] = int(prompt.astype(np.int64).sum())
        return _token(seed, 0, self.prompt_sum[slot])

    def serve_step(self, tokens, active, temperature, seeds, draws):
        out = np.zeros(self.slots, np.uint16)
        for s in range(self.slots):
            if active[s]:
                assert self.busy[s], "stepped a free slot"
                out[s] = _token(seeds[s], draws[s], self.prompt_sum[s])
        return out

    def serve_release(self, slot):
        assert self.busy[slot], "released a free slot"
        self.busy[slot] = False
        self.released.append(slot)


def _requests(n, seed=0):
    rng = np.random.default_rng(seed)
    return [(rng.integers(0, V, rng.integers(1, 9)).astype(np.uint16), int(rng.integers(1, 20)),
             int(rng.integers(0, 2 ** 31))) for _ in range(n)]


def _serve(reqs, slots):
    ex = FakeExecution()
    srv = Server(ex, slots=slots, temperature=1.0)
    ids = [srv.submit(p, m, s) for p, m, s in reqs]
    done = srv.run()
    return ex, [done[i] for i in ids]


@pytest.mark.parametrize("slots", [1, 3, 8])
def test_requests_match_serving_alone(slots):
    reqs = _requests(23)
    ex, got = _serve(reqs, slots)
    for (p, m, s), r in zip(reqs, got):
        _, (alone,) = _serve([(p, m, s)], 1)
        assert r.tokens == alone.tokens and r.finish_reason == alone.finish_reason
    assert ex.max_busy <= slots
    assert len(ex.released) == len(reqs) and not any(ex.busy)


def test_stop_and_length():
    reqs = _requests(40, seed=3)
    _, got = _serve(reqs, 4)
    assert {r.finish_reason for r in got} == {"stop", "length"}
    for (p, m, s), r in zip(reqs, got):
        assert 1 <= len(r.tokens) <= m
        if r.finish_reason == "stop":
            assert r.tokens[-1] == EOS and EOS not in r.tokens[:-1]
        else:
            assert len(r.tokens) == m and EOS not in r.tokens


def test_slots_are_refilled_from_the_queue():
    ex = FakeExecution()
    srv = Server(ex, slots=2, temperature=1.0)
    for p, m, s in _requests(6, seed=5):
        srv.submit(p, m, s)
    busy_seen = []
    while srv.pending():
        srv.step()
        busy_seen.append(sum(ex.busy))
    assert max(busy_seen) <= 2 and ex.max_busy == 2
    assert len(srv.done) == 6 and len(ex.released) == 6


def test_prompt_that_does_not_fit_is_refused():
    ex = FakeExecution()
    srv = Server(ex, slots=2, max_context=16)
    with pytest.raises(EngineError):
        srv.submit(np.arange(10, dtype=np.uint16), 7)
    with pytest.raises(EngineError):
        srv.submit(np.zeros(0, np.uint16), 4)
    assert srv.submit(np.arange(10, dtype=np.uint16), 6) == 0
