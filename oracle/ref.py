"""Test infrastructure: ctypes view of the reference engine's own CPU path.

``oracle/_ref/libmini_mla_ref.so`` is the unmodified reference CPU sources plus
``oracle/ref_harness.cpp``, built by ``oracle/Makefile``. Only tests, the smoke check
and the CPU-baseline leg of ``bench.py`` import this module; the product never does.

Every method names the reference function it drives (file:line in the reference).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libmini_mla_ref.so")
# The same reference sources with sessions on the sm_100a backend through its reference-side
# adapter (`make -C oracle cuda`): the reference's own Execution-API drivers on the GPU.
CUDA_LIB_PATH = os.path.join(_HERE, "_ref", "libmini_mla_ref_cuda.so")

_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int)
_u64p = ctypes.POINTER(ctypes.c_uint64)

_libs = {}


def available(backend: str = "cpu") -> bool:
    return os.path.exists(CUDA_LIB_PATH if backend == "cuda" else LIB_PATH)


def lib(backend: str = "cpu"):
    L = _libs.get(backend)
    if L is None:
        path = CUDA_LIB_PATH if backend == "cuda" else LIB_PATH
        if not os.path.exists(path):
            raise RuntimeError(f"reference oracle not built: {path} (run make -C oracle)")
        L = ctypes.CDLL(path)
        L.ref_last_error.restype = ctypes.c_char_p
        L.ref_session_create.restype = ctypes.c_void_p
        L.ref_session_create.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_float,
                                         ctypes.c_float, ctypes.c_uint64, ctypes.c_int, _f32p]
        L.ref_session_destroy.argtypes = [ctypes.c_void_p]
        L.ref_session_param_count.restype = ctypes.c_int64
        L.ref_session_param_count.argtypes = [ctypes.c_void_p]
        L.ref_session_read.argtypes = [ctypes.c_void_p, ctypes.c_int, _f32p]
        L.ref_session_write.argtypes = [ctypes.c_void_p, ctypes.c_int, _f32p]
        L.ref_session_steps.restype = ctypes.c_uint64
        L.ref_session_steps.argtypes = [ctypes.c_void_p]
        L.ref_session_set_steps.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
        L.ref_forward.argtypes = [ctypes.c_void_p, _u16p, ctypes.c_int, ctypes.c_int, _f32p]
        L.ref_log_probs.argtypes = [ctypes.c_void_p, _u16p, _u16p, _f32p, ctypes.c_int,
                                    ctypes.c_int, _f32p]
        L.ref_zero_grad.argtypes = [ctypes.c_void_p]
        L.ref_accumulate.argtypes = [ctypes.c_void_p, _u16p, _u16p, _f32p, _f32p, ctypes.c_int,
                                     ctypes.c_int, _f64p]
        L.ref_update.argtypes = [ctypes.c_void_p, ctypes.c_float, _f64p]
        L.ref_prefill.argtypes = [ctypes.c_void_p, _u16p, ctypes.c_int, _f32p]
        L.ref_decode.argtypes = [ctypes.c_void_p, ctypes.c_uint16, _f32p]
        L.ref_sample_token.argtypes = [_f32p, ctypes.c_int, _u16p, ctypes.c_int, ctypes.c_float,
                                       ctypes.c_float, ctypes.c_int, ctypes.c_float, _u16p,
                                       ctypes.c_int, _u64p, _u16p]
        L.ref_grpo_objective.argtypes = [ctypes.c_float] * 6 + [_f64p, _f64p, _f32p]
        L.ref_group_advantages.argtypes = [_f32p, ctypes.c_int, ctypes.c_float, _f32p]
        L.ref_completion_batch.argtypes = [_u16p, ctypes.c_int, _u16p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_uint16, _u16p, _u16p, _f32p]
        L.ref_cosine_lr.restype = ctypes.c_float
        L.ref_cosine_lr.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                                    ctypes.c_float, ctypes.c_float]
        for name, rt in (("ref_rng_next", ctypes.c_uint64), ("ref_rng_uniform", ctypes.c_float),
                         ("ref_rng_normal", ctypes.c_float)):
            f = getattr(L, name)
            f.restype = rt
            f.argtypes = [_u64p]
        L.ref_rng_bounded.restype = ctypes.c_uint64
        L.ref_rng_bounded.argtypes = [_u64p, ctypes.c_uint64]
        L.ref_rollout.argtypes = [ctypes.c_void_p, _u16p, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_uint16, ctypes.c_uint16, ctypes.c_uint64,
                                  ctypes.c_float, _u16p, _i32p, _u16p, _u16p, _f32p, _f32p]
        L.ref_dpo_objective.argtypes = [ctypes.c_double] * 4 + [ctypes.c_float, _f64p, _f64p, _f32p, _f32p]
        L.ref_dpo_update.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _u16p, _u16p,
                                     _f32p, ctypes.c_float, ctypes.c_float, _f64p, _f64p, _f64p]
        L.ref_grpo_update.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, _u16p, _u16p, _f32p, _f32p,
                                      _f32p, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                      _f64p, _f64p, _f64p, _i32p, _f32p, _f32p]
        _libs[backend] = L
    return L


def _p(a, t):
    return a.ctypes.data_as(t)


class RefError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"reference error {code}: {message}")
        self.code = code


def _check(rc: int, L=None):
    if rc != 0:
        raise RefError(rc, (L or lib()).ref_last_error().decode())


class Session:
    """Model + optional AdamW Optimizer + ``make_execution("cpu")``
    (src/model/model.cpp:20-75, src/train/optimizer.cpp:53-72, src/infer/inference.cpp:314-329);
    with backend="cuda" the execution is the sm_100a backend's reference-side adapter
    (make_cuda_execution) and the same reference code drives the GPU."""

    def __init__(self, cfg, seed: int, optimizer=None, backend: str = "cpu"):
        L = self.L = lib(backend)
        ints = (ctypes.c_int * 11)(*cfg.int_fields())
        opt = np.asarray(optimizer if optimizer is not None else [0.9, 0.95, 1e-8, 0.1, 1.0],
                         dtype=np.float32)
        self.cfg = cfg
        self.h = L.ref_session_create(ints, cfg.norm_epsilon, cfg.rope_theta, seed,
                                      1 if optimizer is not None else 0, _p(opt, _f32p))
        if not self.h:
            raise RefError(1, L.ref_last_error().decode())
        self.n = int(L.ref_session_param_count(self.h))

    def close(self):
        if self.h:
            self.L.ref_session_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _read(self, which):
        out = np.empty(self.n, np.float32)
        _check(self.L.ref_session_read(self.h, which, _p(out, _f32p)), self.L)
        return out

    def _write(self, which, arr):
        a = np.ascontiguousarray(arr, dtype=np.float32)
        assert a.size == self.n
        _check(self.L.ref_session_write(self.h, which, _p(a, _f32p)), self.L)

    def params(self):
        return self._read(0)

    def grads(self):
        return self._read(1)

    def moments(self):
        return self._read(2), self._read(3)

    def set_params(self, flat):
        self._write(0, flat)

    def set_grads(self, flat):
        self._write(1, flat)

    def set_moments(self, m, v):
        self._write(2, m)
        self._write(3, v)

    @property
    def steps(self):
        return int(self.L.ref_session_steps(self.h))

    @steps.setter
    def steps(self, s):
        self.L.ref_session_set_steps(self.h, s)

    def forward(self, tokens, batch, seq):
        t = np.ascontiguousarray(tokens, np.uint16).reshape(-1)
        out = np.empty((batch * seq, self.cfg.vocab_size), np.float32)
        _check(self.L.ref_forward(self.h, _p(t, _u16p), batch, seq, _p(out, _f32p)), self.L)
        return out

    def log_probs(self, inp, tgt, mask, batch, seq):
        i = np.ascontiguousarray(inp, np.uint16).reshape(-1)
        t = np.ascontiguousarray(tgt, np.uint16).reshape(-1)
        m = np.ascontiguousarray(mask, np.float32).reshape(-1)
        out = np.empty(batch * seq, np.float32)
        _check(self.L.ref_log_probs(self.h, _p(i, _u16p), _p(t, _u16p), _p(m, _f32p), batch, seq,
                                   _p(out, _f32p)), self.L)
        return out

    def zero_grad(self):
        _check(self.L.ref_zero_grad(self.h), self.L)

    def accumulate(self, inp, tgt, mask, coef, batch, seq):
        i = np.ascontiguousarray(inp, np.uint16).reshape(-1)
        t = np.ascontiguousarray(tgt, np.uint16).reshape(-1)
        m = np.ascontiguousarray(mask, np.float32).reshape(-1)
        c = np.ascontiguousarray(coef, np.float32).reshape(-1)
        loss = ctypes.c_double()
        _check(self.L.ref_accumulate(self.h, _p(i, _u16p), _p(t, _u16p), _p(m, _f32p),
                                    _p(c, _f32p), batch, seq, ctypes.byref(loss)), self.L)
        return loss.value

    def update(self, lr):
        norm = ctypes.c_double()
        _check(self.L.ref_update(self.h, lr, ctypes.byref(norm)), self.L)
        return norm.value

    def prefill(self, ids):
        a = np.ascontiguousarray(ids, np.uint16)
        out = np.empty(self.cfg.vocab_size, np.float32)
        _check(self.L.ref_prefill(self.h, _p(a, _u16p), a.size, _p(out, _f32p)), self.L)
        return out

    def decode(self, token):
        out = np.empty(self.cfg.vocab_size, np.float32)
        _check(self.L.ref_decode(self.h, int(token), _p(out, _f32p)), self.L)
        return out

    def rollout(self, prompt, completion_tokens, sequence, eos, pad, seed, temperature=1.0):
        """rollout() of src/train/trainer.cpp:187-213 (restated over the public API)."""
        p = np.ascontiguousarray(prompt, np.uint16)
        toks = np.zeros(max(completion_tokens, 1), np.uint16)
        n = ctypes.c_int()
        inp = np.zeros(sequence, np.uint16)
        tgt = np.zeros(sequence, np.uint16)
        mask = np.zeros(sequence, np.float32)
        old = np.zeros(sequence, np.float32)
        _check(self.L.ref_rollout(self.h, _p(p, _u16p), p.size, completion_tokens, sequence, eos,
                                 pad, seed, temperature, _p(toks, _u16p), ctypes.byref(n),
                                 _p(inp, _u16p), _p(tgt, _u16p), _p(mask, _f32p), _p(old, _f32p)), self.L)
        return dict(tokens=toks[: n.value].copy(), input=inp, target=tgt, mask=mask, old_lp=old)


def grpo_update(policy: Session, reference: Session, group_size, inp, tgt, mask, old_lp, rewards,
                clip, klc, lr):
    """GRPO update body of src/train/trainer.cpp:814-883 (restated over the public API)."""
    n, seq = inp.shape
    i = np.ascontiguousarray(inp, np.uint16)
    t = np.ascontiguousarray(tgt, np.uint16)
    m = np.ascontiguousarray(mask, np.float32)
    o = np.ascontiguousarray(old_lp, np.float32)
    r = np.ascontiguousarray(rewards, np.float32)
    loss, kl, norm = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
    skipped = ctypes.c_int()
    adv = np.zeros(n, np.float32)
    coef = np.zeros((n, seq), np.float32)
    _check(policy.L.ref_grpo_update(policy.h, reference.h, n, group_size, seq, _p(i, _u16p),
                                 _p(t, _u16p), _p(m, _f32p), _p(o, _f32p), _p(r, _f32p), clip,
                                 klc, lr, ctypes.byref(loss), ctypes.byref(kl),
                                 ctypes.byref(norm), ctypes.byref(skipped), _p(adv, _f32p),
                                 _p(coef, _f32p)), policy.L)
    return dict(loss=loss.value, kl=kl.value, grad_norm=norm.value, skipped=bool(skipped.value),
                advantages=adv, coefficients=coef)


def sample_token(logits, rng_state, temperature=1.0, top_p=1.0, top_k=0, repetition_penalty=1.0,
                 history=(), banned=()):
    """sample_token (src/infer/inference.cpp:345-426). Returns (token, new_rng_state)."""
    lg = np.ascontiguousarray(logits, np.float32)
    h = np.ascontiguousarray(history, np.uint16)
    b = np.ascontiguousarray(banned, np.uint16)
    st = ctypes.c_uint64(rng_state)
    out = ctypes.c_uint16()
    _check(lib().ref_sample_token(_p(lg, _f32p), lg.size, _p(h, _u16p), h.size, temperature,
                                  top_p, top_k, repetition_penalty, _p(b, _u16p), b.size,
                                  ctypes.byref(st), ctypes.byref(out)))
    return int(out.value), int(st.value)


def grpo_objective(lp, old, ref, adv, clip, klc):
    loss, kl, coef = ctypes.c_double(), ctypes.c_double(), ctypes.c_float()
    _check(lib().ref_grpo_objective(lp, old, ref, adv, clip, klc, ctypes.byref(loss),
                                    ctypes.byref(kl), ctypes.byref(coef)))
    return loss.value, kl.value, coef.value


def group_advantages(rewards, eps=1e-6):
    r = np.ascontiguousarray(rewards, np.float32)
    out = np.zeros_like(r)
    _check(lib().ref_group_advantages(_p(r, _f32p), r.size, eps, _p(out, _f32p)))
    return out


def completion_batch(prompt, response, seq, pad):
    p = np.ascontiguousarray(prompt, np.uint16)
    r = np.ascontiguousarray(response, np.uint16)
    i = np.zeros(seq, np.uint16)
    t = np.zeros(seq, np.uint16)
    m = np.zeros(seq, np.float32)
    _check(lib().ref_completion_batch(_p(p, _u16p), p.size, _p(r, _u16p), r.size, seq, pad,
                                      _p(i, _u16p), _p(t, _u16p), _p(m, _f32p)))
    return i, t, m


def cosine_lr(done, total, warmup, peak, minimum):
    return float(lib().ref_cosine_lr(done, total, warmup, peak, minimum))


class Rng:
    """The reference Rng (include/mini_mla/rng.hpp:7-35), stepped inside the reference build."""

    def __init__(self, seed):
        self.state = ctypes.c_uint64(seed)

    def next(self):
        return int(lib().ref_rng_next(ctypes.byref(self.state)))

    def uniform(self):
        return float(lib().ref_rng_uniform(ctypes.byref(self.state)))

    def bounded(self, bound):
        return int(lib().ref_rng_bounded(ctypes.byref(self.state), bound))

    def normal(self):
        return float(lib().ref_rng_normal(ctypes.byref(self.state)))


def dpo_objective(chosen, rejected, ref_chosen, ref_rejected, beta):
    """dpo_objective (src/train/trainer.cpp:345-350): (loss, margin, chosen, rejected coefficients)."""
    loss, margin = ctypes.c_double(), ctypes.c_double()
    cc, cr = ctypes.c_float(), ctypes.c_float()
    _check(lib().ref_dpo_objective(chosen, rejected, ref_chosen, ref_rejected, beta, ctypes.byref(loss),
                                   ctypes.byref(margin), ctypes.byref(cc), ctypes.byref(cr)))
    return loss.value, margin.value, cc.value, cr.value


def dpo_update(policy: Session, reference: Session, inp, tgt, mask, beta, lr):
    """DPO update body of src/train/trainer.cpp:765-783 (restated over the public API); pair p is
    rows 2p (chosen) and 2p + 1 (rejected) of [2n, seq] arrays."""
    rows, seq = inp.shape
    n = rows // 2
    i = np.ascontiguousarray(inp, np.uint16)
    t = np.ascontiguousarray(tgt, np.uint16)
    m = np.ascontiguousarray(mask, np.float32)
    loss, norm = ctypes.c_double(), ctypes.c_double()
    margins = np.zeros(n, np.float64)
    _check(policy.L.ref_dpo_update(policy.h, reference.h, n, seq, _p(i, _u16p), _p(t, _u16p), _p(m, _f32p),
                                   beta, lr, ctypes.byref(loss), ctypes.byref(norm), _p(margins, _f64p)),
           policy.L)
    return dict(loss=loss.value, grad_norm=norm.value, margins=margins)
