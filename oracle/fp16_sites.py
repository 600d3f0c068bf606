"""Test infrastructure: where the fp16 compute of the teacher-forced pass loses accuracy.

The numpy restatement's forward (oracle/mla_oracle.py, Model::forward of
src/model/model.cpp:76-155) with each place where the CUDA path rounds to fp16 switched on
or off: the activations that feed tensor-core products (the attention RMSNorm output `h`,
the normalised q and kv latents `cq`/`ckv`, q, k, v, the softmax P, the attention output, the
FFN input `h2`, the SwiGLU output `gated`) and every weight matrix. Prints the mean and
maximum |log-prob - fp32 log-prob| over 8 x 256 random tokens of the 35.8M model (frozen
reference init, seed 1) with every site rounded, and with chosen sites exact. This is how the
FFN was chosen for the three-term product.

    python -m oracle.fp16_sites
"""
from __future__ import annotations

import sys
import time

import numpy as np

from cpp_inference_train_engine_b200.config import MLA36M
from oracle import mla_oracle as O

F32 = np.float32
ACTS = ["h", "cq", "q", "ckv", "v", "k", "P", "ao", "h2", "gated"]
WEIGHTS = ["w_dq", "w_dkv", "w_uq", "w_uk", "w_uv", "w_o", "w_gate", "w_up", "w_down"]


def _round(on, name, a):
    return a.astype(np.float16).astype(F32) if name in on else a


def forward_logits(c, P, tokens, batch, seq, on):
    """Model::forward with fp16 rounding at the sites in `on`."""
    x = P.embedding[tokens].astype(F32)
    cos, sin = O.rope_table(c, np.arange(seq))
    cos, sin = np.tile(cos, (batch, 1)), np.tile(sin, (batch, 1))
    mask = np.tril(np.ones((seq, seq), bool))
    sc = F32(1) / np.sqrt(F32(c.qk_dim))
    for layer in range(c.n_layers):
        def w(n):
            t = P.layer(layer, n)
            return _round(on, n, t) if n.startswith("w_") else t
        h = _round(on, "h", O.rmsnorm(x, w("attn_norm"), c.norm_epsilon))
        cq = _round(on, "cq", O.rmsnorm(h @ w("w_dq"), w("q_norm"), c.norm_epsilon))
        q = _round(on, "q", O.rope(cq @ w("w_uq"), cos, sin, c.n_heads, c.qk_dim, c.head_dim_nope))
        kvp = h @ w("w_dkv")
        ckv = _round(on, "ckv", O.rmsnorm(kvp[:, :c.kv_lora_rank].copy(), w("kv_norm"), c.norm_epsilon))
        kr = O.rope(kvp[:, c.kv_lora_rank:].copy(), cos, sin, 1, c.head_dim_rope, 0)
        kn = ckv @ w("w_uk")
        v = _round(on, "v", ckv @ w("w_uv"))
        k = np.zeros((x.shape[0], c.n_heads * c.qk_dim), F32)
        for hh in range(c.n_heads):
            k[:, hh * c.qk_dim:hh * c.qk_dim + c.head_dim_nope] = kn[:, hh * c.head_dim_nope:(hh + 1) * c.head_dim_nope]
            k[:, hh * c.qk_dim + c.head_dim_nope:(hh + 1) * c.qk_dim] = kr
        k = _round(on, "k", k)
        ao = np.zeros((x.shape[0], c.attn_width), F32)
        qd, vd = c.qk_dim, c.head_dim_value
        for b in range(batch):
            r = slice(b * seq, (b + 1) * seq)
            for hh in range(c.n_heads):
                s = (q[r][:, hh * qd:(hh + 1) * qd] @ k[r][:, hh * qd:(hh + 1) * qd].T) * sc
                s = np.where(mask, s, -np.inf).astype(F32)
                p = np.exp(s - s.max(1, keepdims=True))
                den = p.sum(1, keepdims=True, dtype=F32)
                ao[r][:, hh * vd:(hh + 1) * vd] = (_round(on, "P", p) @ v[r][:, hh * vd:(hh + 1) * vd]) / den
        res = (_round(on, "ao", ao) @ w("w_o") + x).astype(F32)
        h2 = _round(on, "h2", O.rmsnorm(res, w("ffn_norm"), c.norm_epsilon))
        gated = _round(on, "gated", O.swiglu(h2 @ w("w_gate"), h2 @ w("w_up")))
        x = (gated @ w("w_down") + res).astype(F32)
    fin = O.rmsnorm(x, P.final_norm, c.norm_epsilon)
    return (fin @ P.embedding.T).astype(F32)


def log_probs(logits, tgt):
    m = logits.max(1, keepdims=True)
    z = np.log(np.exp((logits - m).astype(np.float64)).sum(1))
    return logits[np.arange(len(tgt)), tgt] - m[:, 0] - z


def main(argv=None):
    c = MLA36M
    P = O.Params(c, O.init_params(c, 1))
    rng = np.random.default_rng(0)
    B, S = 8, 256
    ids = rng.integers(0, c.vocab_size, (B, S + 1))
    tok, tgt = ids[:, :S].reshape(-1), ids[:, 1:].reshape(-1)
    exact = log_probs(forward_logits(c, P, tok, B, S, set()), tgt)
    every = set(ACTS + WEIGHTS)
    for keep in [set(), {"h2"}, {"h2", "h", "ckv", "cq"},
                 {"h2", "h", "ckv", "cq", "w_dq", "w_dkv", "w_uq", "w_uk", "w_uv"},
                 {"h2", "w_gate", "w_up"}, {"h2", "gated", "w_down"}]:
        t0 = time.time()
        d = np.abs(log_probs(forward_logits(c, P, tok, B, S, every - keep), tgt) - exact)
        print(f"exact {sorted(keep)}: mean {d.mean():.4e} max {d.max():.4e} ({time.time() - t0:.0f} s)", flush=True)


if __name__ == "__main__":
    sys.exit(main())
