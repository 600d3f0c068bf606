"""Host-side mirror of the reference engine's Execution interface over the C ABI of
``libmm_cuda.so`` (include/mm_cuda.h).

Names, argument meanings and error behaviour follow the reference:
``make_execution(model, optimizer, backend, precision)`` (src/infer/inference.cpp:314-329),
``Execution.forward / log_probabilities / accumulate / zero_grad / update / step /
prefill / decode / synchronize_to_host`` (include/mini_mla/execution.hpp:28-61), failures
raised as :class:`EngineError` carrying the reference's ErrorCode (result.hpp:9-16).
The batched entry points (``rollout``, ``grpo_step``, ``prefill_batch``,
``decode_batch``) are the B200 forms of ``rollout()`` and the GRPO update body
(src/train/trainer.cpp:187-213, 814-891).

There is no CPU fallback: without the built library or a CUDA device every call fails.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from .config import AdamWConfig, ModelConfig

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmm_cuda.so")

ERROR_NAMES = {1: "invalid_argument", 2: "io_error", 3: "unsupported", 4: "out_of_memory",
               5: "gpu_error", 6: "numerical_error"}

_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_vp = ctypes.c_void_p


class EngineError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code
        self.name = ERROR_NAMES.get(code, str(code))


class ModelDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "vocab_size", "max_sequence_length", "n_layers", "d_model", "n_heads", "head_dim_nope",
        "head_dim_rope", "head_dim_value", "q_lora_rank", "kv_lora_rank", "d_ff")] + [
        ("norm_epsilon", ctypes.c_float), ("rope_theta", ctypes.c_float)]

    @staticmethod
    def of(cfg: ModelConfig) -> "ModelDesc":
        return ModelDesc(*cfg.int_fields(), cfg.norm_epsilon, cfg.rope_theta)


class AdamWDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_float) for n in
                ("beta1", "beta2", "epsilon", "weight_decay", "clip_norm")]


class StepResult(ctypes.Structure):
    _fields_ = [("loss", ctypes.c_double), ("kl", ctypes.c_double),
                ("grad_norm", ctypes.c_double), ("skipped", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


_lib = None


def lib():
    """Loads libmm_cuda.so (fails loudly when it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise EngineError(3, f"CUDA backend not built: {LIB_PATH} "
                             "(run python -m cpp_inference_train_engine_b200.build)")
    L = ctypes.CDLL(LIB_PATH)
    sig = {
        "mm_model_parameter_count": (ctypes.c_int64, [ctypes.POINTER(ModelDesc)]),
        "mm_model_init_params": (ctypes.c_int, [ctypes.POINTER(ModelDesc), ctypes.c_uint64, _f32p]),
        "mm_cosine_learning_rate": (ctypes.c_float, [ctypes.c_uint64, ctypes.c_uint64,
                                                     ctypes.c_uint64, ctypes.c_float,
                                                     ctypes.c_float]),
        "mm_cuda_create": (ctypes.c_int, [ctypes.POINTER(ModelDesc), ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(AdamWDesc), ctypes.POINTER(_vp)]),
        "mm_cuda_destroy": (None, [_vp]),
        "mm_cuda_last_error": (ctypes.c_size_t, [_vp, ctypes.c_char_p, ctypes.c_size_t]),
        "mm_cuda_upload_params": (ctypes.c_int, [_vp, _f32p, _f32p, _f32p, ctypes.c_uint64]),
        "mm_cuda_download": (ctypes.c_int, [_vp, _f32p, _f32p, _f32p, _f32p, _u64p]),
        "mm_cuda_forward_logits": (ctypes.c_int, [_vp, _u16p, ctypes.c_int, ctypes.c_int, _f32p]),
        "mm_cuda_log_probs": (ctypes.c_int, [_vp, _u16p, _u16p, ctypes.c_int, ctypes.c_int, _f32p]),
        "mm_cuda_zero_grad": (ctypes.c_int, [_vp]),
        "mm_cuda_accumulate": (ctypes.c_int, [_vp, _u16p, _u16p, _f32p, ctypes.c_int, ctypes.c_int,
                                              _f64p]),
        "mm_cuda_update": (ctypes.c_int, [_vp, ctypes.c_float, _f64p]),
        "mm_cuda_prefill_batch": (ctypes.c_int, [_vp, _u16p, ctypes.c_int, ctypes.c_int, _f32p]),
        "mm_cuda_decode_batch": (ctypes.c_int, [_vp, _u16p, ctypes.c_int, _f32p]),
        "mm_cuda_sample": (ctypes.c_int, [_vp, _f32p, ctypes.c_int, ctypes.c_float, _u64p, _i32p,
                                          _u16p]),
        "mm_cuda_rollout": (ctypes.c_int, [_vp, _u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_uint16, ctypes.c_uint16, _u64p,
                                           ctypes.c_float, _u16p, _i32p, _u16p, _u16p, _f32p,
                                           _f32p]),
        "mm_cuda_grpo_coefficients": (ctypes.c_int, [_vp, _f32p, _f32p, _f32p, _f32p, _f32p,
                                                     ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                     ctypes.c_int64, ctypes.c_float,
                                                     ctypes.c_float, _f32p, _f32p, _f64p, _f64p]),
        "mm_cuda_grpo_step": (ctypes.c_int, [_vp, _vp, _u16p, _u16p, _f32p, _f32p, _f32p,
                                             ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int64, ctypes.c_float, ctypes.c_float,
                                             ctypes.c_float, ctypes.POINTER(StepResult)]),
        "mm_cuda_dpo_step": (ctypes.c_int, [_vp, _vp, _u16p, _u16p, _f32p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int64, ctypes.c_float, ctypes.c_float,
                                            ctypes.POINTER(StepResult), ctypes.POINTER(ctypes.c_double)]),
        "mm_cuda_serve_open": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int]),
        "mm_cuda_serve_admit": (ctypes.c_int, [_vp, ctypes.c_int, _u16p, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_float, ctypes.c_uint64, _u16p, _f32p]),
        "mm_cuda_serve_step": (ctypes.c_int, [_vp, _u16p, _i32p, ctypes.c_float, _u64p, _i32p, _u16p, _f32p]),
        "mm_cuda_serve_release": (ctypes.c_int, [_vp, ctypes.c_int]),
        "mm_cuda_nccl_unique_id": (ctypes.c_int, [ctypes.c_char_p]),
        "mm_cuda_init_comm": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_char_p]),
        "mm_cuda_kernel_launches": (ctypes.c_int64, [_vp]),
        "mm_cuda_gemm_f16": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp,
                                            ctypes.c_int64, ctypes.c_int, _vp, ctypes.c_int64,
                                            ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int,
                                            ctypes.c_float, _vp, ctypes.c_int64, ctypes.c_int]),
        "mm_cuda_profile": (ctypes.c_int, [_vp, ctypes.c_int, _f64p, _i64p, _f64p]),
        "mm_cuda_decode_trace": (ctypes.c_int, [_vp, ctypes.c_int, _u64p, ctypes.c_int, _i32p]),
        "mm_cuda_stream": (ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
        "mm_cuda_decode_attention": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int64, _vp, ctypes.c_int,
                                                    ctypes.c_int, ctypes.c_float, _vp]),
        "mm_cuda_profile_gemm_shapes": (ctypes.c_int64, [_vp, ctypes.c_char_p, ctypes.c_int64]),
        "mm_cuda_selftest_wait_timeout": (ctypes.c_int, [_vp, ctypes.c_uint32]),
        "mm_cuda_bench_gemm": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              _vp, ctypes.c_int64, ctypes.c_int, _vp, ctypes.c_int64,
                                              ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int,
                                              ctypes.POINTER(ctypes.c_float)]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


def parameter_count(cfg: ModelConfig) -> int:
    return int(lib().mm_model_parameter_count(ctypes.byref(ModelDesc.of(cfg))))


def init_params(cfg: ModelConfig, seed: int) -> np.ndarray:
    """Model::create's initial weights (src/model/model.cpp:20-75), flat registry order."""
    out = np.empty(parameter_count(cfg), np.float32)
    rc = lib().mm_model_init_params(ctypes.byref(ModelDesc.of(cfg)), seed, _p(out, _f32p))
    if rc:
        raise EngineError(rc, "invalid model configuration")
    return out


def cosine_learning_rate(done, total, warmup, peak, minimum):
    return float(lib().mm_cosine_learning_rate(done, total, warmup, peak, minimum))


PROFILE_TAGS = ("prefill", "decode", "sample", "logprob", "backward", "adamw", "allreduce", "prep",
                "k_gemm", "k_decode_attention", "k_flash_fwd", "k_flash_bwd", "k_sample",
                "k_logsoftmax", "k_adamw", "k_other")


class CudaExecution:
    """One device context (Execution of backend "cuda"). ``trainable`` allocates
    gradients and AdamW moments (an Execution built with an Optimizer)."""

    def __init__(self, cfg: ModelConfig, device: int = 0, trainable: bool = False,
                 optimizer: AdamWConfig | None = None):
        L = lib()
        self.cfg = cfg
        self.trainable = trainable
        h = _vp()
        opt = AdamWDesc(*(optimizer or AdamWConfig()).as_list())
        rc = L.mm_cuda_create(ctypes.byref(ModelDesc.of(cfg)), device, 1 if trainable else 0,
                              ctypes.byref(opt), ctypes.byref(h))
        self.h = h
        if rc:
            msg = self._error()
            L.mm_cuda_destroy(h)
            self.h = None
            raise EngineError(rc, msg)
        self.n_params = parameter_count(cfg)

    # ------------------------------------------------------------------ plumbing
    def _error(self) -> str:
        buf = ctypes.create_string_buffer(4096)
        lib().mm_cuda_last_error(self.h, buf, 4096)
        return buf.value.decode(errors="replace")

    def _check(self, rc):
        if rc:
            raise EngineError(rc, self._error())

    def close(self):
        if getattr(self, "h", None):
            lib().mm_cuda_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def kernel_launches(self) -> int:
        return int(lib().mm_cuda_kernel_launches(self.h))

    @property
    def stream(self) -> int:
        s = _vp()
        self._check(lib().mm_cuda_stream(self.h, ctypes.byref(s)))
        return s.value or 0

    # ------------------------------------------------------------------ state
    def upload(self, params, m=None, v=None, steps: int = 0):
        p = np.ascontiguousarray(params, np.float32)
        if p.size != self.n_params:
            raise EngineError(1, f"expected {self.n_params} parameters, got {p.size}")
        m = None if m is None else np.ascontiguousarray(m, np.float32)
        v = None if v is None else np.ascontiguousarray(v, np.float32)
        self._check(lib().mm_cuda_upload_params(self.h, _p(p, _f32p), _p(m, _f32p),
                                                _p(v, _f32p), steps))

    def synchronize_to_host(self, params=True, grads=False, moments=False):
        """Execution::synchronize_to_host: returns dict of flat arrays and the step count."""
        out = {}
        arr = lambda: np.empty(self.n_params, np.float32)
        P = arr() if params else None
        G = arr() if grads else None
        M = arr() if moments else None
        V = arr() if moments else None
        steps = ctypes.c_uint64()
        self._check(lib().mm_cuda_download(self.h, _p(P, _f32p), _p(G, _f32p), _p(M, _f32p),
                                           _p(V, _f32p), ctypes.byref(steps)))
        if params:
            out["params"] = P
        if grads:
            out["grads"] = G
        if moments:
            out["m"], out["v"] = M, V
        out["steps"] = int(steps.value)
        return out

    # ------------------------------------------------------------------ Execution
    def forward(self, tokens, batch: int, seq: int):
        t = np.ascontiguousarray(tokens, np.uint16).reshape(-1)
        out = np.empty((batch * seq, self.cfg.vocab_size), np.float32)
        self._check(lib().mm_cuda_forward_logits(self.h, _p(t, _u16p), batch, seq,
                                                 _p(out, _f32p)))
        return out

    def log_probabilities(self, inp, tgt, batch: int, seq: int):
        i = np.ascontiguousarray(inp, np.uint16).reshape(-1)
        t = np.ascontiguousarray(tgt, np.uint16).reshape(-1)
        out = np.empty(batch * seq, np.float32)
        self._check(lib().mm_cuda_log_probs(self.h, _p(i, _u16p), _p(t, _u16p), batch, seq,
                                            _p(out, _f32p)))
        return out

    def zero_grad(self):
        self._check(lib().mm_cuda_zero_grad(self.h))

    def accumulate(self, inp, tgt, coefficients, batch: int, seq: int) -> float:
        i = np.ascontiguousarray(inp, np.uint16).reshape(-1)
        t = np.ascontiguousarray(tgt, np.uint16).reshape(-1)
        c = np.ascontiguousarray(coefficients, np.float32).reshape(-1)
        loss = ctypes.c_double()
        self._check(lib().mm_cuda_accumulate(self.h, _p(i, _u16p), _p(t, _u16p), _p(c, _f32p),
                                             batch, seq, ctypes.byref(loss)))
        return loss.value

    def update(self, learning_rate: float) -> float:
        n = ctypes.c_double()
        self._check(lib().mm_cuda_update(self.h, learning_rate, ctypes.byref(n)))
        return n.value

    def step(self, jobs, learning_rate: float):
        """Execution::step (inference.cpp:282-302): jobs = [(inp, tgt, coef, batch, seq)]."""
        if not jobs or not np.isfinite(learning_rate) or learning_rate < 0:
            raise EngineError(1, "Invalid training step")
        for j in jobs:
            if not np.all(np.isfinite(np.asarray(j[2], np.float32))):
                raise EngineError(1, "Invalid gradient batch")
        loss = sum(self.accumulate(*j) for j in jobs)
        return {"loss": loss, "gradient_norm": self.update(learning_rate)}

    # ------------------------------------------------------------------ decode sessions
    def prefill_batch(self, prompts):
        p = np.ascontiguousarray(prompts, np.uint16)
        if p.ndim == 1:
            p = p[None, :]
        out = np.empty((p.shape[0], self.cfg.vocab_size), np.float32)
        self._check(lib().mm_cuda_prefill_batch(self.h, _p(p, _u16p), p.shape[0], p.shape[1],
                                                _p(out, _f32p)))
        return out

    def decode_batch(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint16).reshape(-1)
        out = np.empty((t.size, self.cfg.vocab_size), np.float32)
        self._check(lib().mm_cuda_decode_batch(self.h, _p(t, _u16p), t.size, _p(out, _f32p)))
        return out

    def prefill(self, ids):
        """Execution::prefill for one prompt (batch of one)."""
        return self.prefill_batch(np.asarray(ids, np.uint16)[None, :])[0]

    def decode(self, token):
        return self.decode_batch(np.array([token], np.uint16))[0]

    def sample(self, logits, temperature, seeds, draw_index=None):
        lg = np.ascontiguousarray(logits, np.float32)
        if lg.ndim == 1:
            lg = lg[None, :]
        if lg.shape[1] != self.cfg.vocab_size:
            raise EngineError(1, "Invalid sampler logits: width must equal the vocabulary")
        s = np.ascontiguousarray(seeds, np.uint64).reshape(-1)
        if s.size != lg.shape[0] or (draw_index is not None and np.size(draw_index) != s.size):
            raise EngineError(1, "one seed (and draw index) per row")
        d = None if draw_index is None else np.ascontiguousarray(draw_index, np.int32)
        out = np.empty(lg.shape[0], np.uint16)
        self._check(lib().mm_cuda_sample(self.h, _p(lg, _f32p), lg.shape[0], temperature,
                                         _p(s, _u64p), _p(d, _i32p), _p(out, _u16p)))
        return out

    def rollout(self, prompts, completion_tokens, sequence, seeds, temperature=1.0,
                with_batches=True):
        """rollout() for every prompt row at once (trainer.cpp:187-213)."""
        p = np.ascontiguousarray(prompts, np.uint16)
        n, P = p.shape
        s = np.ascontiguousarray(seeds, np.uint64)
        toks = np.empty((n, completion_tokens), np.uint16)
        lens = np.empty(n, np.int32)
        inp = tgt = mask = old = None
        if with_batches:
            inp = np.empty((n, sequence), np.uint16)
            tgt = np.empty((n, sequence), np.uint16)
            mask = np.empty((n, sequence), np.float32)
            old = np.empty((n, sequence), np.float32)
        self._check(lib().mm_cuda_rollout(self.h, _p(p, _u16p), n, P, completion_tokens,
                                          sequence, self.cfg.eos_id, self.cfg.pad_id,
                                          _p(s, _u64p), temperature, _p(toks, _u16p),
                                          _p(lens, _i32p), _p(inp, _u16p), _p(tgt, _u16p),
                                          _p(mask, _f32p), _p(old, _f32p)))
        out = {"tokens": toks, "lengths": lens}
        if with_batches:
            out.update(input=inp, target=tgt, mask=mask, old_lp=old)
        return out

    def grpo_coefficients(self, lp, old, ref, mask, rewards, group_size, n_total, clip, klc):
        lp, old, ref, mask = [np.ascontiguousarray(a, np.float32) for a in (lp, old, ref, mask)]
        r = np.ascontiguousarray(rewards, np.float32)
        n, seq = lp.shape
        coef = np.empty_like(lp)
        adv = np.empty(n, np.float32)
        loss, kl = ctypes.c_double(), ctypes.c_double()
        self._check(lib().mm_cuda_grpo_coefficients(
            self.h, _p(lp, _f32p), _p(old, _f32p), _p(ref, _f32p), _p(mask, _f32p), _p(r, _f32p),
            n, seq, group_size, n_total, clip, klc, _p(coef, _f32p), _p(adv, _f32p),
            ctypes.byref(loss), ctypes.byref(kl)))
        return {"coefficients": coef, "advantages": adv, "loss": loss.value, "kl": kl.value}

    def grpo_step(self, reference: "CudaExecution", inp, tgt, mask, old_lp, rewards, group_size,
                  n_total=None, clip=0.2, klc=0.04, learning_rate=1e-5):
        i = np.ascontiguousarray(inp, np.uint16)
        t = np.ascontiguousarray(tgt, np.uint16)
        m = np.ascontiguousarray(mask, np.float32)
        o = np.ascontiguousarray(old_lp, np.float32)
        r = np.ascontiguousarray(rewards, np.float32)
        n, seq = i.shape
        res = StepResult()
        self._check(lib().mm_cuda_grpo_step(self.h, reference.h, _p(i, _u16p), _p(t, _u16p),
                                            _p(m, _f32p), _p(o, _f32p), _p(r, _f32p), n, seq,
                                            group_size, n_total or n, clip, klc, learning_rate,
                                            ctypes.byref(res)))
        return {"loss": res.loss, "kl": res.kl, "grad_norm": res.grad_norm,
                "skipped": bool(res.skipped)}

    def dpo_step(self, reference: "CudaExecution", inp, tgt, mask, beta=0.1, n_total=None,
                 learning_rate=1e-5):
        """One DPO update (mm_cuda_dpo_step) over preference pairs: rows 2p (chosen) and 2p + 1
        (rejected) of [2n, seq] arrays. Returns loss, mean margin, pre-clip gradient norm and the
        per-pair margins."""
        i = np.ascontiguousarray(inp, np.uint16)
        t = np.ascontiguousarray(tgt, np.uint16)
        m = np.ascontiguousarray(mask, np.float32)
        rows, seq = i.shape
        if rows % 2 or t.shape != i.shape or m.shape != i.shape:
            raise EngineError(1, "preference pairs need [2n, seq] input, target and mask")
        n = rows // 2
        res = StepResult()
        margins = np.empty(n, np.float64)
        self._check(lib().mm_cuda_dpo_step(self.h, reference.h, _p(i, _u16p), _p(t, _u16p), _p(m, _f32p), n,
                                           seq, n_total or n, beta, learning_rate, ctypes.byref(res),
                                           margins.ctypes.data_as(ctypes.POINTER(ctypes.c_double))))
        return {"loss": res.loss, "margin": res.kl, "grad_norm": res.grad_norm, "margins": margins}

    # ------------------------------------------------------------------ serving
    def serve_open(self, slots: int, max_context: int):
        """Opens a continuous-batching session of `slots` requests (mm_cuda_serve_open)."""
        self._check(lib().mm_cuda_serve_open(self.h, slots, max_context))

    def serve_admit(self, slot, prompt, max_new, temperature=0.0, seed=0, with_logits=False):
        """Prefills `prompt` into `slot`; returns the first token (and its logits)."""
        p = np.ascontiguousarray(prompt, np.uint16).reshape(-1)
        first = np.zeros(1, np.uint16)
        lg = np.empty(self.cfg.vocab_size, np.float32) if with_logits else None
        self._check(lib().mm_cuda_serve_admit(self.h, slot, _p(p, _u16p), p.size, max_new, temperature,
                                              int(seed), _p(first, _u16p), _p(lg, _f32p)))
        return (int(first[0]), lg) if with_logits else int(first[0])

    def serve_step(self, tokens, active, temperature, seeds, draw_index, with_logits=False):
        """One decode step of the active slots; returns the next token of every slot."""
        t = np.ascontiguousarray(tokens, np.uint16)
        a = np.ascontiguousarray(active, np.int32)
        s = np.ascontiguousarray(seeds, np.uint64)
        d = np.ascontiguousarray(draw_index, np.int32)
        nxt = np.zeros(t.size, np.uint16)
        lg = np.empty((t.size, self.cfg.vocab_size), np.float32) if with_logits else None
        self._check(lib().mm_cuda_serve_step(self.h, _p(t, _u16p), _p(a, _i32p), temperature, _p(s, _u64p),
                                             _p(d, _i32p), _p(nxt, _u16p), _p(lg, _f32p)))
        return (nxt, lg) if with_logits else nxt

    def serve_release(self, slot: int):
        self._check(lib().mm_cuda_serve_release(self.h, slot))

    # ------------------------------------------------------------------ data parallel
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        rc = lib().mm_cuda_nccl_unique_id(buf)
        if rc:
            raise EngineError(rc, "ncclGetUniqueId failed")
        return buf.raw

    def init_comm(self, rank: int, world: int, uid: bytes):
        self._check(lib().mm_cuda_init_comm(self.h, rank, world, uid))

    # ------------------------------------------------------------------ kernels / timing
    def gemm(self, M, N, K, a_ptr, lda, a_mn, b_ptr, ldb, b_mn, out_ptr, ldc, out_kind,
             alpha=1.0, residual_ptr=None, ldr=0, bf16=False):
        self._check(lib().mm_cuda_gemm_f16(self.h, M, N, K, a_ptr, lda, int(a_mn), b_ptr, ldb,
                                           int(b_mn), out_ptr, ldc, out_kind, alpha,
                                           residual_ptr, ldr, int(bf16)))

    def bench_gemm(self, reps, M, N, K, a_ptr, lda, a_mn, b_ptr, ldb, b_mn, out_ptr, ldc, out_kind):
        """Device milliseconds per launch of `reps` back-to-back launches of one product,
        replayed from a CUDA graph (mm_cuda_bench_gemm)."""
        ms = ctypes.c_float(0.0)
        self._check(lib().mm_cuda_bench_gemm(self.h, reps, M, N, K, a_ptr, lda, int(a_mn), b_ptr, ldb,
                                             int(b_mn), out_ptr, ldc, out_kind, ctypes.byref(ms)))
        return float(ms.value)

    def decode_attention(self, q_ptr, cache_ptr, cache_seq_stride, pos_ptr, batch, splits, scale,
                         out_ptr):
        """Kernel-level latent decode attention on device pointers (mm_cuda_kernels.h)."""
        self._check(lib().mm_cuda_decode_attention(self.h, q_ptr, cache_ptr, cache_seq_stride,
                                                   pos_ptr, batch, splits, scale, out_ptr))

    def selftest_wait_timeout(self, polls: int = 1 << 12):
        """Runs the bounded-wait failure path (mm_cuda_selftest_wait_timeout): raises
        EngineError(gpu_error) and leaves this execution unusable."""
        self._check(lib().mm_cuda_selftest_wait_timeout(self.h, polls))

    def gemm_shapes(self):
        """Per-shape GEMM timing collected while profiling: list of dicts."""
        n = lib().mm_cuda_profile_gemm_shapes(self.h, None, 0)
        if n < 0:
            raise EngineError(-n, self._error())
        buf = ctypes.create_string_buffer(int(n) + 1)
        lib().mm_cuda_profile_gemm_shapes(self.h, buf, n + 1)
        out = []
        for line in buf.value.decode().splitlines():
            parts = dict(p.split("=") for p in line.split() if "=" in p)
            out.append({"shape": " ".join(p for p in line.split() if "=" not in p),
                        "calls": int(parts["calls"]), "ms": float(parts["ms"]),
                        "tflops": float(parts["tflops"])})
        return sorted(out, key=lambda r: -r["ms"])

    def decode_trace(self, enable: int = -1):
        """Phase trace of the fused decode step (mm_cuda_decode_trace): with enable 1/0 turns it
        on/off; returns the last traced step's phase durations in microseconds."""
        buf = np.zeros(320, np.uint64)
        n = ctypes.c_int32()
        self._check(lib().mm_cuda_decode_trace(self.h, enable, _p(buf, _u64p), buf.size, ctypes.byref(n)))
        t = buf[:min(n.value, 128)].astype(np.int64)
        t = t[t > 0]
        return (np.diff(t) / 1e3).tolist() if t.size > 1 else []

    def decode_trace_raw(self):
        """The raw timestamps (ns) of the last traced fused decode step: [0, 128) start, barriers,
        end; [128, 256) per GEMM phase g: producer start, accumulator ready, epilogue done;
        [256, 320) per layer l (4 l): CTA 0 warp 0's first attention item starts, its queries are
        ready, its cache tiles are done, its row is merged."""
        buf = np.zeros(320, np.uint64)
        n = ctypes.c_int32()
        self._check(lib().mm_cuda_decode_trace(self.h, -1, _p(buf, _u64p), buf.size, ctypes.byref(n)))
        return buf[:n.value].astype(np.int64)

    def profile(self, enable: int = -1):
        """{tag: (device ms, launches, algorithmic work)}; see PROFILE_TAGS."""
        ms = (ctypes.c_double * 16)()
        calls = (ctypes.c_int64 * 16)()
        work = (ctypes.c_double * 16)()
        self._check(lib().mm_cuda_profile(self.h, enable, ms, calls, work))
        return {PROFILE_TAGS[i]: (ms[i], int(calls[i]), work[i]) for i in range(16)}


def make_execution(cfg: ModelConfig, params, optimizer: AdamWConfig | None = None,
                   backend: str = "cuda", precision: str = "fp16", device: int = 0, moments=None,
                   steps: int = 0) -> CudaExecution:
    """make_execution (src/infer/inference.cpp:314-329) for backend "cuda": fp16 tensor-core
    compute over fp32 master weights. `optimizer` present = a training execution."""
    if backend != "cuda" or precision not in ("fp16", "fp32"):
        raise EngineError(3, "Select cuda/fp16")
    e = CudaExecution(cfg, device=device, trainable=optimizer is not None, optimizer=optimizer)
    m, v = moments if moments is not None else (None, None)
    e.upload(params, m, v, steps)
    return e
