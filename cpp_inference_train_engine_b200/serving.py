"""Continuous-batching generation on the batched latent-cache decode.

The reference serves one request at a time: `InferenceEngine::generate_tokens`
(src/infer/inference.cpp:469-579) prefills the prompt, then per token samples with the
request's `Rng(seed)`, stops after `<|eos|>` or `max_new_tokens`, and decodes the sampled
token when another is due. `Server` runs many such requests together on one execution: every
slot of an `mm_cuda_serve_*` session holds one request, queued requests are admitted into
slots as others finish, and each engine step decodes every active slot in one batched pass
(the same kernels as the rollout). Per request the token sequence is the one
`generate_tokens` produces with top_p = 1, top_k = 0, repetition penalty 1 and no stop
strings: draw i of the request's own Rng, whatever else shares the batch.
"""
from __future__ import annotations

import collections
from dataclasses import dataclass, field

import numpy as np

from .engine import CudaExecution, EngineError


@dataclass
class Request:
    rid: int
    prompt: np.ndarray
    max_new_tokens: int
    seed: int = 0
    tokens: list = field(default_factory=list)
    finish_reason: str = ""


class Server:
    """Admits queued requests into free slots and steps all active slots together.

    `temperature` is the session's (0 = greedy); `eos` ends a request after emitting it
    (default: the model's end-of-sequence id, vocab_size - 6)."""

    def __init__(self, execution: CudaExecution, slots: int, max_context: int | None = None,
                 temperature: float = 0.0, eos: int | None = None):
        cfg = execution.cfg
        self.ex = execution
        self.slots = slots
        self.max_context = max_context or cfg.max_sequence_length
        self.temperature = float(temperature)
        self.eos = cfg.vocab_size - 6 if eos is None else int(eos)
        self.queue: collections.deque[Request] = collections.deque()
        self.slot_req: list[Request | None] = [None] * slots
        self.done: dict[int, Request] = {}
        self._next_id = 0
        execution.serve_open(slots, self.max_context)

    def submit(self, prompt, max_new_tokens: int, seed: int = 0) -> int:
        p = np.ascontiguousarray(prompt, np.uint16).reshape(-1)
        if p.size < 1 or max_new_tokens < 1 or p.size + max_new_tokens > self.max_context:
            raise EngineError(1, "Prompt plus requested tokens exceeds context")
        r = Request(self._next_id, p, int(max_new_tokens), int(seed))
        self._next_id += 1
        self.queue.append(r)
        return r.rid

    def _finish(self, slot: int, reason: str):
        r = self.slot_req[slot]
        r.finish_reason = reason
        self.done[r.rid] = r
        self.slot_req[slot] = None
        self.ex.serve_release(slot)

    def _after_token(self, slot: int, token: int):
        r = self.slot_req[slot]
        r.tokens.append(int(token))
        if token == self.eos:
            self._finish(slot, "stop")
        elif len(r.tokens) >= r.max_new_tokens:
            self._finish(slot, "length")

    def step(self) -> list[int]:
        """Admits what fits, then one batched decode step. Returns the ids finished by it."""
        before = set(self.done)
        for s in range(self.slots):
            if self.slot_req[s] is None and self.queue:
                r = self.queue.popleft()
                self.slot_req[s] = r
                first = self.ex.serve_admit(s, r.prompt, r.max_new_tokens, self.temperature, r.seed)
                self._after_token(s, first)
        active = np.array([r is not None for r in self.slot_req], np.int32)
        if active.any():
            tokens = np.array([r.tokens[-1] if r else 0 for r in self.slot_req], np.uint16)
            seeds = np.array([r.seed if r else 0 for r in self.slot_req], np.uint64)
            draws = np.array([len(r.tokens) if r else 0 for r in self.slot_req], np.int32)
            nxt = self.ex.serve_step(tokens, active, self.temperature, seeds, draws)
            for s in range(self.slots):
                if active[s]:
                    self._after_token(s, int(nxt[s]))
        return sorted(set(self.done) - before)

    def pending(self) -> int:
        return len(self.queue) + sum(r is not None for r in self.slot_req)

    def run(self) -> dict[int, Request]:
        """Steps until every submitted request has finished."""
        while self.pending():
            self.step()
        return self.done
