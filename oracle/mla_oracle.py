"""Test infrastructure: a CPU restatement, in numpy, of the reference engine's GRPO hot
path. It is the checker for the CUDA path, never part of it; only tests, the smoke check
and bench.py's CPU-baseline leg import it.

Parity pins: tests/test_oracle.py checks every function here against the reference's
own golden vectors (tests/golden/attention_sync_oracle.npz, re-packed from
docs/verification/attention-sync/oracle) and against the reference CPU build
(oracle/_ref, see oracle/Makefile).

Arithmetic follows the reference: float32 tensors and float32 matrix products; float64
exactly where the reference switches to double (the log-softmax normaliser, the
sampler's weights, the GRPO objective, the optimiser's global norm and bias
corrections). Each function cites the reference lines it restates.
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32
MASK64 = (1 << 64) - 1


# ---------------------------------------------------------------- Rng (rng.hpp:7-35)
class Rng:
    """splitmix64 (include/mini_mla/rng.hpp:10-15)."""

    def __init__(self, seed: int):
        self.state = seed & MASK64

    def next(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & MASK64
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
        return z ^ (z >> 31)

    def uniform(self) -> float:
        """rng.hpp:16-18: ((next >> 40) + 0.5) / 2^24, exact in float32."""
        return float((F32(self.next() >> 40) + F32(0.5)) / F32(16777216.0))

    def bounded(self, bound: int) -> int:
        """rng.hpp:19-27 (rejection below (2^64 - bound) % bound)."""
        if bound == 0:
            return 0
        threshold = ((1 << 64) - bound) % bound
        while True:
            r = self.next()
            if r >= threshold:
                return r % bound

    def normal(self) -> float:
        """rng.hpp:28-31, Box-Muller in float32."""
        u1 = F32(self.uniform())
        u2 = F32(self.uniform())
        return float(np.sqrt(F32(-2.0) * np.log(u1)) * np.cos(F32(2.0 * np.pi).astype(F32) * u2))


def counter_uniform(seed: int, k: int) -> float:
    """Draw k (0-based) of Rng(seed).uniform(): splitmix64 is counter based, so draw k is
    mix(seed + (k+1)*gamma). This is the form the device sampler uses."""
    r = Rng((seed + k * 0x9E3779B97F4A7C15) & MASK64)
    return r.uniform()


# ---------------------------------------------------------------- model registry
def init_params(cfg, seed: int):
    """Model::create (src/model/model.cpp:20-75): registry order, norms = 1, matrices
    N(0, 0.02^2) with w_o / w_down scaled by 1/sqrt(2L). Returns a list of arrays."""
    rng = Rng(seed)
    out = []
    resid = F32(0.02) / np.sqrt(F32(2 * cfg.n_layers))
    for name, (r, c), role in cfg.parameter_shapes():
        if role == "norm_scale":
            out.append(np.ones((r, c), F32))
            continue
        scale = resid if (name.endswith("w_o") or name.endswith("w_down")) else F32(0.02)
        vals = np.array([rng.normal() for _ in range(r * c)], F32) * F32(scale)
        out.append(vals.reshape(r, c))
    return out


def split_params(cfg, flat):
    """Flat registry-order vector -> list of [rows, cols] views."""
    out, off = [], 0
    for _, (r, c), _ in cfg.parameter_shapes():
        out.append(np.asarray(flat[off:off + r * c], F32).reshape(r, c))
        off += r * c
    return out


class Params:
    NAMES = ["attn_norm", "w_dq", "q_norm", "w_uq", "w_dkv", "kv_norm", "w_uk", "w_uv", "w_o",
             "ffn_norm", "w_gate", "w_up", "w_down"]

    def __init__(self, cfg, tensors):
        self.cfg = cfg
        self.t = tensors
        self.embedding = tensors[0]
        self.final_norm = tensors[1]

    def layer(self, l, name):
        return self.t[2 + l * 13 + Params.NAMES.index(name)]


# ---------------------------------------------------------------- ops (ops.cpp)
def rmsnorm(x, w, eps):
    """ops::rmsnorm (src/model/ops.cpp:33-45)."""
    ss = np.sum(x * x, axis=-1, dtype=F32, keepdims=True)
    inv = F32(1.0) / np.sqrt(ss / F32(x.shape[-1]) + F32(eps))
    return (x * inv * w.reshape(-1)).astype(F32)


def rmsnorm_backward(x, w, dy, eps):
    """ops::rmsnorm_backward (src/model/ops.cpp:46-64): returns (dx, dw)."""
    w = w.reshape(-1)
    sq = np.sum(x * x, axis=-1, dtype=F32, keepdims=True)
    dot = np.sum(dy * w * x, axis=-1, dtype=F32, keepdims=True)
    inv = F32(1.0) / np.sqrt(sq / F32(x.shape[-1]) + F32(eps))
    corr = dot * inv * inv * inv / F32(x.shape[-1])
    dx = dy * w * inv - x * corr
    dw = np.sum(dy * x * inv, axis=0, dtype=F32)
    return dx.astype(F32), dw.reshape(1, -1)


def sigmoid(x):
    """ops::sigmoid (src/model/ops.cpp:65-70), the two-branch stable form."""
    x = x.astype(F32)
    e = np.exp(-np.abs(x))
    return np.where(x >= 0, F32(1) / (F32(1) + e), e / (F32(1) + e)).astype(F32)


def swiglu(g, u):
    """ops::swiglu (src/model/ops.cpp:71-77)."""
    return (g * sigmoid(g) * u).astype(F32)


def swiglu_backward(g, u, dy):
    """ops::swiglu_backward (src/model/ops.cpp:78-87): returns (dgate, dup)."""
    s = sigmoid(g)
    return (dy * u * (s + g * s * (F32(1) - s))).astype(F32), (dy * g * s).astype(F32)


def rope_table(cfg, positions):
    """Angles of ops::rope (src/model/ops.cpp:88-108): for pair j (even), position t:
    angle = t * theta^(-j / rope_width), float32; returns (cos, sin) [T, rope/2]."""
    w = cfg.head_dim_rope
    j = np.arange(0, w, 2)
    freq = np.array([np.power(F32(cfg.rope_theta), -F32(jj) / F32(w)) for jj in j], F32)
    ang = (np.asarray(positions, F32)[:, None] * freq[None, :]).astype(F32)
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def rope(x, cos, sin, heads, width, begin, inverse=False):
    """ops::rope on rows of x [T, heads*width]: adjacent pairs (begin+j, begin+j+1)."""
    x = x.copy()
    if inverse:
        sin = -sin
    for h in range(heads):
        a = x[:, h * width + begin:h * width + begin + cos.shape[1] * 2:2].copy()
        b = x[:, h * width + begin + 1:h * width + begin + cos.shape[1] * 2:2].copy()
        x[:, h * width + begin:h * width + begin + cos.shape[1] * 2:2] = a * cos - b * sin
        x[:, h * width + begin + 1:h * width + begin + cos.shape[1] * 2:2] = a * sin + b * cos
    return x.astype(F32)


def causal_attention(q, k, v, heads, d, dv):
    """ops::attention for one sequence (src/model/ops.cpp:109-142): q,k [T, H*d],
    v [T, H*dv]; softmax in float32 over j <= i. Returns (P [H,T,T], out [T, H*dv])."""
    T = q.shape[0]
    scale = F32(1.0) / np.sqrt(F32(d))
    P = np.zeros((heads, T, T), F32)
    out = np.zeros((T, heads * dv), F32)
    mask = np.tril(np.ones((T, T), bool))
    for h in range(heads):
        s = (q[:, h * d:(h + 1) * d] @ k[:, h * d:(h + 1) * d].T) * scale
        s = np.where(mask, s, -np.inf).astype(F32)
        s = np.exp(s - s.max(axis=1, keepdims=True))
        s = s / s.sum(axis=1, keepdims=True, dtype=F32)
        P[h] = s
        out[:, h * dv:(h + 1) * dv] = s @ v[:, h * dv:(h + 1) * dv]
    return P, out


def causal_attention_backward(q, k, v, P, dy, heads, d, dv):
    """ops::attention_backward (src/model/ops.cpp:143-172)."""
    scale = F32(1.0) / np.sqrt(F32(d))
    dq, dk, dvv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    for h in range(heads):
        p = P[h]
        g = dy[:, h * dv:(h + 1) * dv]
        s = g @ v[:, h * dv:(h + 1) * dv].T
        dvv[:, h * dv:(h + 1) * dv] = p.T @ g
        dot = np.sum(s * p, axis=1, keepdims=True, dtype=F32)
        s = p * (s - dot)
        dq[:, h * d:(h + 1) * d] = (s @ k[:, h * d:(h + 1) * d]) * scale
        dk[:, h * d:(h + 1) * d] = (s.T @ q[:, h * d:(h + 1) * d]) * scale
    return dq, dk, dvv


def weighted_nll(logits, targets, coef, want_grad=False):
    """ops::weighted_nll (src/model/ops.cpp:173-210): float32 row max, float64 sum of
    exp, lp = -(log z + max - l_t) rounded to float32; grad = coef*(softmax - onehot).
    Returns (loss, log_probs, grad or None)."""
    lg = logits.astype(F32)
    mx = lg.max(axis=1)
    ex = np.exp((lg - mx[:, None]).astype(F32).astype(np.float64))
    z = ex.sum(axis=1)
    tl = lg[np.arange(lg.shape[0]), targets].astype(np.float64)
    nll = np.log(z) + mx.astype(np.float64) - tl
    loss = float(np.sum(np.asarray(coef, np.float64) * nll))
    grad = None
    if want_grad:
        sm = (ex / z[:, None]).astype(F32)
        sm[np.arange(lg.shape[0]), targets] -= F32(1)
        grad = (np.asarray(coef, F32)[:, None] * sm).astype(F32)
    return loss, (-nll).astype(F32), grad


# ---------------------------------------------------------------- model forward/backward
class Forward:
    """Model::forward (src/model/model.cpp:76-155) with its tape, batch of B sequences."""

    def __init__(self, cfg, P: Params, tokens, batch, seq):
        c = cfg
        self.cfg, self.P, self.B, self.S = cfg, P, batch, seq
        self.tokens = np.asarray(tokens).reshape(-1).astype(np.int64)
        x = P.embedding[self.tokens].astype(F32)
        self.emb = x
        cos, sin = rope_table(c, np.arange(seq))
        cos, sin = np.tile(cos, (batch, 1)), np.tile(sin, (batch, 1))
        self.cos, self.sin = cos, sin
        self.tape = []
        for l in range(c.n_layers):
            w = lambda n: P.layer(l, n)
            t = {"x": x}
            t["h"] = rmsnorm(x, w("attn_norm"), c.norm_epsilon)
            t["raw_cq"] = t["h"] @ w("w_dq")
            t["cq"] = rmsnorm(t["raw_cq"], w("q_norm"), c.norm_epsilon)
            t["q"] = rope(t["cq"] @ w("w_uq"), cos, sin, c.n_heads, c.qk_dim, c.head_dim_nope)
            kvp = t["h"] @ w("w_dkv")
            t["raw_ckv"] = kvp[:, :c.kv_lora_rank].copy()
            t["ckv"] = rmsnorm(t["raw_ckv"], w("kv_norm"), c.norm_epsilon)
            t["k_rope"] = rope(kvp[:, c.kv_lora_rank:].copy(), cos, sin, 1, c.head_dim_rope, 0)
            k_nope = t["ckv"] @ w("w_uk")
            t["v"] = t["ckv"] @ w("w_uv")
            k = np.zeros((x.shape[0], c.n_heads * c.qk_dim), F32)
            for h in range(c.n_heads):
                k[:, h * c.qk_dim:h * c.qk_dim + c.head_dim_nope] = \
                    k_nope[:, h * c.head_dim_nope:(h + 1) * c.head_dim_nope]
                k[:, h * c.qk_dim + c.head_dim_nope:(h + 1) * c.qk_dim] = t["k_rope"]
            t["k"] = k
            Ps, ao = [], np.zeros((x.shape[0], c.attn_width), F32)
            for b in range(batch):
                r = slice(b * seq, (b + 1) * seq)
                p, o = causal_attention(t["q"][r], k[r], t["v"][r], c.n_heads, c.qk_dim,
                                        c.head_dim_value)
                Ps.append(p)
                ao[r] = o
            t["P"], t["attn_out"] = Ps, ao
            t["residual"] = (ao @ w("w_o") + x).astype(F32)
            t["h2"] = rmsnorm(t["residual"], w("ffn_norm"), c.norm_epsilon)
            t["gate"] = t["h2"] @ w("w_gate")
            t["up"] = t["h2"] @ w("w_up")
            t["gated"] = swiglu(t["gate"], t["up"])
            x = (t["gated"] @ w("w_down") + t["residual"]).astype(F32)
            self.tape.append(t)
        self.out = x
        self.final = rmsnorm(x, P.final_norm, c.norm_epsilon)
        self.logits = (self.final @ P.embedding.T).astype(F32)

    def backward(self, g):
        """Model::backward (src/model/model.cpp:168-245). Returns grads in registry order."""
        c, P = self.cfg, self.P
        grads = [np.zeros_like(a) for a in P.t]
        gi = lambda l, n: 2 + l * 13 + Params.NAMES.index(n)
        dh = g @ P.embedding
        grads[0] += g.T @ self.final
        dy, grads[1] = rmsnorm_backward(self.out, P.final_norm, dh, c.norm_epsilon)
        for l in reversed(range(c.n_layers)):
            t = self.tape[l]
            w = lambda n: P.layer(l, n)
            grads[gi(l, "w_down")] += t["gated"].T @ dy
            dgated = dy @ w("w_down").T
            dg, du = swiglu_backward(t["gate"], t["up"], dgated)
            grads[gi(l, "w_gate")] += t["h2"].T @ dg
            grads[gi(l, "w_up")] += t["h2"].T @ du
            dh2 = dg @ w("w_gate").T + du @ w("w_up").T
            dres, dwn = rmsnorm_backward(t["residual"], w("ffn_norm"), dh2, c.norm_epsilon)
            grads[gi(l, "ffn_norm")] += dwn
            dres = dres + dy
            grads[gi(l, "w_o")] += t["attn_out"].T @ dres
            dao = dres @ w("w_o").T
            dq = np.zeros_like(t["q"])
            dk = np.zeros_like(t["k"])
            dv = np.zeros_like(t["v"])
            for b in range(self.B):
                r = slice(b * self.S, (b + 1) * self.S)
                a, bb, cc = causal_attention_backward(t["q"][r], t["k"][r], t["v"][r], t["P"][b],
                                                      dao[r], c.n_heads, c.qk_dim,
                                                      c.head_dim_value)
                dq[r], dk[r], dv[r] = a, bb, cc
            dq = rope(dq, self.cos, self.sin, c.n_heads, c.qk_dim, c.head_dim_nope, inverse=True)
            dkn = np.zeros((dk.shape[0], c.n_heads * c.head_dim_nope), F32)
            drope = np.zeros((dk.shape[0], c.head_dim_rope), F32)
            for h in range(c.n_heads):
                dkn[:, h * c.head_dim_nope:(h + 1) * c.head_dim_nope] = \
                    dk[:, h * c.qk_dim:h * c.qk_dim + c.head_dim_nope]
                drope += dk[:, h * c.qk_dim + c.head_dim_nope:(h + 1) * c.qk_dim]
            drope = rope(drope, self.cos, self.sin, 1, c.head_dim_rope, 0, inverse=True)
            grads[gi(l, "w_uk")] += t["ckv"].T @ dkn
            grads[gi(l, "w_uv")] += t["ckv"].T @ dv
            dckv = dkn @ w("w_uk").T + dv @ w("w_uv").T
            dkvraw, dwkv = rmsnorm_backward(t["raw_ckv"], w("kv_norm"), dckv, c.norm_epsilon)
            grads[gi(l, "kv_norm")] += dwkv
            dkvp = np.concatenate([dkvraw, drope], axis=1)
            grads[gi(l, "w_dkv")] += t["h"].T @ dkvp
            dhh = dkvp @ w("w_dkv").T
            grads[gi(l, "w_uq")] += t["cq"].T @ dq
            dcq = dq @ w("w_uq").T
            draw, dwq = rmsnorm_backward(t["raw_cq"], w("q_norm"), dcq, c.norm_epsilon)
            grads[gi(l, "q_norm")] += dwq
            grads[gi(l, "w_dq")] += t["h"].T @ draw
            dhh = dhh + draw @ w("w_dq").T
            dx, dwa = rmsnorm_backward(t["x"], w("attn_norm"), dhh, c.norm_epsilon)
            grads[gi(l, "attn_norm")] += dwa
            dy = (dx + dres).astype(F32)
        np.add.at(grads[0], self.tokens, dy)
        return grads


def log_probabilities(cfg, P, inp, tgt, batch, seq):
    """CpuExecution::log_probabilities (src/infer/inference.cpp:197-207)."""
    f = Forward(cfg, P, inp, batch, seq)
    _, lp, _ = weighted_nll(f.logits, np.asarray(tgt).reshape(-1).astype(np.int64),
                            np.zeros(batch * seq))
    return lp


def accumulate(cfg, P, inp, tgt, coef, batch, seq):
    """CpuExecution::accumulate (src/infer/inference.cpp:208-222): (loss, grads)."""
    f = Forward(cfg, P, inp, batch, seq)
    loss, _, g = weighted_nll(f.logits, np.asarray(tgt).reshape(-1).astype(np.int64),
                              np.asarray(coef).reshape(-1), want_grad=True)
    return loss, f.backward(g)


# ---------------------------------------------------------------- AdamW (optimizer.cpp)
def adamw_step(cfg, params, grads, m, v, steps, lr, opt):
    """Optimizer::step, AdamW branch (src/train/optimizer.cpp:105-161). Arrays are lists in
    registry order, updated in place. Returns (pre-clip norm, new step count)."""
    b1, b2, eps, wd, clip = [F32(x) for x in opt]
    sq = 0.0
    for g in grads:
        sq += float(np.sum(g.astype(np.float64) ** 2))
    norm = math.sqrt(sq)
    gs = F32(min(1.0, float(clip) / max(norm, 1e-30))) if clip > 0 else F32(1)
    steps += 1
    bc1 = F32(1.0 - math.pow(float(b1), steps))
    bc2 = F32(1.0 - math.pow(float(b2), steps))
    roles = [r for _, _, r in cfg.parameter_shapes()]
    lr = F32(lr)
    for k in range(len(params)):
        decay = F32(0) if roles[k] == "norm_scale" else wd
        g = grads[k] * gs
        m[k][...] = b1 * m[k] + (F32(1) - b1) * g
        v[k][...] = b2 * v[k] + (F32(1) - b2) * g * g
        params[k][...] = params[k] * (F32(1) - lr * decay) - \
            lr * (m[k] / bc1) / (np.sqrt(v[k] / bc2) + eps)
    return norm, steps


def cosine_learning_rate(done, total, warmup, peak, minimum):
    """cosine_learning_rate (src/train/optimizer.cpp:162-173)."""
    if warmup and done < warmup:
        return float(F32(peak) * F32(done + 1) / F32(warmup))
    if total <= warmup:
        return float(peak)
    t = min(max((done - min(done, warmup)) / (total - warmup), 0.0), 1.0)
    mn = F32(minimum)
    one_minus = float(F32(1) - mn)  # float arithmetic in the reference, then double
    return float(F32(peak) * F32(float(mn) + one_minus * 0.5 * (1 + math.cos(math.pi * t))))


# ---------------------------------------------------------------- GRPO (trainer.cpp)
def grpo_objective(lp, old, ref, adv, clip, klc):
    """grpo_objective (src/train/trainer.cpp:351-370): (loss, kl, float32 coefficient),
    or None when the reference rejects the token (|lp-old| > 80 or |ref-lp| > 80)."""
    lp, old, ref, adv, clip, klc = [float(F32(x)) for x in (lp, old, ref, adv, clip, klc)]
    if abs(float(F32(lp - old))) > 80 or abs(float(F32(ref - lp))) > 80:
        return None
    ratio = math.exp(lp - old)
    clipped = min(max(ratio, 1.0 - clip), 1.0 + clip)
    delta = ref - lp
    ed = math.exp(delta)
    kl = ed - delta - 1
    obj = -min(ratio * adv, clipped * adv) + klc * kl
    # 1 + clip and 1 - clip are float sums in the reference (trainer.cpp:363)
    active = ratio <= float(F32(1.0 + clip)) if adv >= 0 else ratio >= float(F32(1.0 - clip))
    coef = (ratio * adv if active else 0.0) + klc * (ed - 1)
    if not math.isfinite(obj) or abs(coef) > float(np.finfo(F32).max):
        return None
    # the objective hands back the coefficient as a float (trainer.cpp:368-369)
    return obj, kl, float(F32(coef))


# ---------------------------------------------------------------- DPO (trainer.cpp)
def dpo_objective(chosen, rejected, ref_chosen, ref_rejected, beta):
    """dpo_objective (src/train/trainer.cpp:345-350): (loss, margin, chosen and rejected
    float32 coefficients); the loss is the stable softplus of -beta * margin in double."""
    margin = (chosen - rejected) - (ref_chosen - ref_rejected)
    z = float(F32(beta)) * margin
    loss = max(-z, 0.0) + math.log1p(math.exp(-abs(z)))
    scale = F32(beta) * _sigmoid_scalar(-z)
    return loss, margin, float(scale), float(-scale)


def _sigmoid_scalar(x):
    """ops::sigmoid (src/model/ops.cpp:65-70) on one float, with the float exponential
    taken as the correctly rounded value of the double one."""
    x = float(F32(x))
    if x >= 0:
        return F32(1) / (F32(1) + F32(math.exp(-x)))
    e = F32(math.exp(x))
    return e / (F32(1) + e)


def dpo_coefficients(lp, ref_lp, mask, beta):
    """The DPO coefficient loop (trainer.cpp:765-783 with preference_objective :107-121) over
    pairs [2n, S] (rows 2p chosen, 2p + 1 rejected): (loss, margins, float32 coefficients)."""
    n = lp.shape[0] // 2
    coef = np.zeros_like(mask, dtype=F32)
    loss, margins = 0.0, []
    for p in range(n):
        c, r = 2 * p, 2 * p + 1
        sums = [float(np.sum(lp[c][mask[c] != 0], dtype=np.float64)), float(np.sum(lp[r][mask[r] != 0], dtype=np.float64)),
                float(np.sum(ref_lp[c][mask[c] != 0], dtype=np.float64)),
                float(np.sum(ref_lp[r][mask[r] != 0], dtype=np.float64))]
        lo, margin, cc, cr = dpo_objective(sums[0], sums[1], sums[2], sums[3], beta)
        loss += lo / n
        margins.append(margin)
        coef[c] = mask[c] * (F32(cc) / F32(n))
        coef[r] = mask[r] * (F32(cr) / F32(n))
    return loss, np.array(margins), coef


def group_advantages(rewards, eps=1e-6):
    """group_advantages (src/train/trainer.cpp:371-385): population std in double."""
    r = [float(F32(x)) for x in rewards]
    mean = sum(r) / len(r)
    sq = sum((x - mean) * (x - mean) for x in r)
    scale = math.sqrt(sq / len(r)) + float(F32(eps))
    return np.array([(x - mean) / scale for x in r], F32)


def completion_batch(prompt, response, seq, pad):
    """completion_batch (src/train/trainer.cpp:386-408)."""
    ids = list(prompt) + list(response)
    if not prompt or not response or len(ids) > seq + 1:
        raise ValueError("Completion sample exceeds context or has an empty prompt/response")
    inp = np.full(seq, pad, np.uint16)
    tgt = np.full(seq, pad, np.uint16)
    mask = np.zeros(seq, F32)
    for i in range(len(ids) - 1):
        inp[i], tgt[i] = ids[i], ids[i + 1]
        mask[i] = 1 if i + 1 >= len(prompt) else 0
    return inp, tgt, mask


def grpo_coefficients(lp, old, ref, mask, advantages, clip, klc, n_total=None):
    """Coefficient assembly of src/train/trainer.cpp:827-846 over rollouts [N, S]:
    coef = nll_coefficient / (N * supervised_i); loss/kl summed in double. ``n_total``
    replaces N when these rows are one data-parallel shard of a larger step."""
    N = lp.shape[0] if n_total is None else int(n_total)
    coef = np.zeros_like(lp, dtype=F32)
    loss = kl = 0.0
    for i in range(lp.shape[0]):
        sup = int(np.count_nonzero(mask[i] == 1))
        den = float(N * sup)
        for t in np.nonzero(mask[i])[0]:
            o = grpo_objective(lp[i, t], old[i, t], ref[i, t], advantages[i], clip, klc)
            if o is None:
                raise ValueError("Invalid or unbounded GRPO token statistics")
            loss += o[0] / den
            kl += o[1] / den
            # float coefficient / double denominator, rounded to float (trainer.cpp:842-843)
            coef[i, t] = F32(o[2] / den)
    return loss, kl, coef


# ---------------------------------------------------------------- sampling (inference.cpp)
def sample_token(logits, u, temperature):
    """sample_token without penalties/bans (src/infer/inference.cpp:345-426). `u` is the
    float uniform draw of the reference Rng for this call (unused when greedy)."""
    lg = np.asarray(logits, F32)
    if temperature == 0:
        return int(np.argmax(lg))  # lowest index among maxima (inference.cpp:363-375)
    order = np.lexsort((np.arange(lg.size), -lg.astype(np.float64)))
    p = np.exp((lg[order] - lg[order[0]]).astype(F32).astype(np.float64) / float(F32(temperature)))
    total = 0.0
    for x in p:  # sequential double sum (inference.cpp:407-413)
        total += x
    kept, count = 0.0, 0
    while True:  # top_p = 1 keeps the prefix whose sum reaches the total (:414-418)
        kept += p[count]
        count += 1
        if not (count < len(p) and kept < total):
            break
    draw = float(u) * kept
    for i in range(count):
        draw -= p[i]
        if draw <= 0:
            return int(order[i])
    return int(order[count - 1])


# ---------------------------------------------------------------- cached decode
class Decoder:
    """CpuDecoder with absorbed projections (src/infer/inference.cpp:28-174): latent
    cache ckv [pos, kv_rank] and rotated rope key [pos, rope] per layer."""

    def __init__(self, cfg, P: Params):
        self.cfg, self.P = cfg, P
        c = cfg
        self.lat = [np.zeros((c.max_sequence_length, c.kv_lora_rank), F32)
                    for _ in range(c.n_layers)]
        self.kr = [np.zeros((c.max_sequence_length, c.head_dim_rope), F32)
                   for _ in range(c.n_layers)]
        self.pos = 0
        # prepare_projections (inference.cpp:28-46): per head W_uv[:,h] @ W_o[h rows].
        self.outp = []
        for l in range(c.n_layers):
            uv, wo = P.layer(l, "w_uv"), P.layer(l, "w_o")
            dv = c.head_dim_value
            self.outp.append(np.concatenate(
                [uv[:, h * dv:(h + 1) * dv] @ wo[h * dv:(h + 1) * dv] for h in range(c.n_heads)],
                axis=0).astype(F32))

    def prefill(self, ids):
        f = Forward(self.cfg, self.P, ids, 1, len(ids))
        for l in range(self.cfg.n_layers):
            self.lat[l][:len(ids)] = f.tape[l]["ckv"]
            self.kr[l][:len(ids)] = f.tape[l]["k_rope"]
        self.pos = len(ids)
        return f.logits[-1].copy()

    def decode(self, token):
        c, P = self.cfg, self.P
        x = P.embedding[int(token)][None, :].astype(F32)
        cos, sin = rope_table(c, [self.pos])
        n = self.pos + 1
        scale = F32(1.0) / np.sqrt(F32(c.qk_dim))
        for l in range(c.n_layers):
            w = lambda nm: P.layer(l, nm)
            h = rmsnorm(x, w("attn_norm"), c.norm_epsilon)
            cq = rmsnorm(h @ w("w_dq"), w("q_norm"), c.norm_epsilon)
            q = rope(cq @ w("w_uq"), cos, sin, c.n_heads, c.qk_dim, c.head_dim_nope)
            kvp = h @ w("w_dkv")
            self.lat[l][self.pos] = rmsnorm(kvp[:, :c.kv_lora_rank], w("kv_norm"),
                                            c.norm_epsilon)[0]
            self.kr[l][self.pos] = rope(kvp[:, c.kv_lora_rank:].copy(), cos, sin, 1,
                                        c.head_dim_rope, 0)[0]
            ctx = np.zeros((1, c.n_heads * c.kv_lora_rank), F32)
            uk = w("w_uk")
            for hh in range(c.n_heads):
                qh = q[0, hh * c.qk_dim:(hh + 1) * c.qk_dim]
                ql = uk[:, hh * c.head_dim_nope:(hh + 1) * c.head_dim_nope] @ qh[:c.head_dim_nope]
                s = self.lat[l][:n] @ ql + self.kr[l][:n] @ qh[c.head_dim_nope:]
                s = (s * scale).astype(F32)
                s = np.exp(s - s.max()).astype(F32)
                s = s / s.sum(dtype=F32)
                ctx[0, hh * c.kv_lora_rank:(hh + 1) * c.kv_lora_rank] = s @ self.lat[l][:n]
            res = (ctx @ self.outp[l] + x).astype(F32)
            h2 = rmsnorm(res, w("ffn_norm"), c.norm_epsilon)
            x = (swiglu(h2 @ w("w_gate"), h2 @ w("w_up")) @ w("w_down") + res).astype(F32)
        self.pos += 1
        return (rmsnorm(x, P.final_norm, c.norm_epsilon) @ P.embedding.T)[0].astype(F32)
