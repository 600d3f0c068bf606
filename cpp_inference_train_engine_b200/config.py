"""Model and run configuration, mirroring the reference's ``ModelConfig``
(include/mini_mla/model_config.hpp:5-19, src/model/config.cpp:7-48) and the GRPO
options the hot path reads from ``TrainOptions`` (include/mini_mla/trainer.hpp:5-28)."""
from __future__ import annotations

import dataclasses
import json


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    vocab_size: int = 264
    max_sequence_length: int = 64
    n_layers: int = 2
    d_model: int = 32
    n_heads: int = 2
    head_dim_nope: int = 12
    head_dim_rope: int = 4
    head_dim_value: int = 16
    q_lora_rank: int = 16
    kv_lora_rank: int = 8
    d_ff: int = 64
    norm_epsilon: float = 1e-5
    rope_theta: float = 10000.0

    @property
    def qk_dim(self) -> int:
        return self.head_dim_nope + self.head_dim_rope

    @property
    def kv_width(self) -> int:
        return self.kv_lora_rank + self.head_dim_rope

    @property
    def attn_width(self) -> int:
        return self.n_heads * self.head_dim_value

    # Special ids occupy the top 8 vocabulary slots (src/infer/tokenizer.cpp:11-12):
    # pad = V-8, bos = V-7, eos = V-6.
    @property
    def pad_id(self) -> int:
        return self.vocab_size - 8

    @property
    def eos_id(self) -> int:
        return self.vocab_size - 6

    def int_fields(self):
        return [self.vocab_size, self.max_sequence_length, self.n_layers, self.d_model,
                self.n_heads, self.head_dim_nope, self.head_dim_rope, self.head_dim_value,
                self.q_lora_rank, self.kv_lora_rank, self.d_ff]

    def parameter_shapes(self):
        """Registry order and shapes of Model::create (src/model/model.cpp:40-63)."""
        d, H = self.d_model, self.n_heads
        out = [("token_embedding", (self.vocab_size, d), "token_embedding"),
               ("final_norm", (1, d), "norm_scale")]
        for l in range(self.n_layers):
            p = f"layers.{l}."
            out += [
                (p + "attn.norm", (1, d), "norm_scale"),
                (p + "attn.w_dq", (d, self.q_lora_rank), "hidden_matrix"),
                (p + "attn.q_norm", (1, self.q_lora_rank), "norm_scale"),
                (p + "attn.w_uq", (self.q_lora_rank, H * self.qk_dim), "hidden_matrix"),
                (p + "attn.w_dkv", (d, self.kv_width), "hidden_matrix"),
                (p + "attn.kv_norm", (1, self.kv_lora_rank), "norm_scale"),
                (p + "attn.w_uk", (self.kv_lora_rank, H * self.head_dim_nope), "hidden_matrix"),
                (p + "attn.w_uv", (self.kv_lora_rank, self.attn_width), "hidden_matrix"),
                (p + "attn.w_o", (self.attn_width, d), "hidden_matrix"),
                (p + "ffn.norm", (1, d), "norm_scale"),
                (p + "ffn.w_gate", (d, self.d_ff), "hidden_matrix"),
                (p + "ffn.w_up", (d, self.d_ff), "hidden_matrix"),
                (p + "ffn.w_down", (self.d_ff, d), "hidden_matrix"),
            ]
        return out

    def parameter_count(self) -> int:
        """ModelConfig::parameter_count (src/model/config.cpp:7-19)."""
        return sum(r * c for _, (r, c), _ in self.parameter_shapes())

    @staticmethod
    def from_json(obj) -> "ModelConfig":
        if isinstance(obj, str):
            with open(obj) as f:
                obj = json.load(f)
        names = {f.name for f in dataclasses.fields(ModelConfig)}
        return ModelConfig(**{k: v for k, v in obj.items() if k in names})


# config/tiny-test.json of the reference.
TINY = ModelConfig()
# config/mla36m-v1.json of the reference: 35,763,840 parameters.
MLA36M = ModelConfig(vocab_size=16384, max_sequence_length=2048, n_layers=10, d_model=512,
                     n_heads=8, head_dim_nope=48, head_dim_rope=16, head_dim_value=64,
                     q_lora_rank=192, kv_lora_rank=128, d_ff=1360)


# The scaled MLA model of the multi-GPU GRPO workload: 24 blocks, width 2048, 16 heads, query
# rank 768, kv rank 512, SwiGLU 5632, tied 32,768-token vocabulary, context 2048. Its head
# widths are this backend's choice (nope 96 + rope 32 = value 128, so query/key and value
# heads have the same width): 1,144,651,776 parameters. The reference's validator caps
# models at 1e9 parameters (src/model/config.cpp:44-46); this backend does not.
MLA1B = ModelConfig(vocab_size=32768, max_sequence_length=2048, n_layers=24, d_model=2048,
                    n_heads=16, head_dim_nope=96, head_dim_rope=32, head_dim_value=128,
                    q_lora_rank=768, kv_lora_rank=512, d_ff=5632)


@dataclasses.dataclass(frozen=True)
class AdamWConfig:
    """OptimizerConfig defaults (include/mini_mla/optimizer.hpp:5-14)."""
    beta1: float = 0.9
    beta2: float = 0.95
    epsilon: float = 1e-8
    weight_decay: float = 0.1
    clip_norm: float = 1.0

    def as_list(self):
        return [self.beta1, self.beta2, self.epsilon, self.weight_decay, self.clip_norm]
