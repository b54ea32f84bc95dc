"""Model configuration for the QuantaWeave-B200 sparse-MoE decoder.

The field names, defaults and validation of the first fourteen fields follow the reference's
``QuantaWeaveConfig`` (``src/quantweave_moe_model.py:15-48``) so that a reference ``config.json`` loads
unchanged and reproduces the reference layout (LayerNorm, learned absolute positions, biased MHA).

The remaining fields are additions needed by the benchmark configurations and by the B200 engine:

* ``norm_type``: ``"layernorm"`` (reference) or ``"rmsnorm"``;
* ``position_embedding``: ``"learned"`` (reference) or ``"rope"``;
* ``kv_heads``: key/value heads for grouped-query attention (``None`` = ``attention_heads``, i.e. MHA);
* ``attention_bias``: biases on the QKV and output projections (reference: True);
* ``rope_theta`` and ``norm_eps``;
* ``init_std``: ``None`` keeps torch's default module initialisation (reference behaviour); a float
  draws every matrix from N(0, init_std).
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, fields
from pathlib import Path
from typing import Optional


@dataclass
class QuantaWeaveConfig:
    vocab_size: int = 7168
    hidden_size: int = 64
    layers: int = 2
    ffn_size: int = 128
    num_experts: int = 184
    top_k: int = 1
    attention_heads: int = 4
    max_sequence_length: int = 256
    router_aux_loss_coef: float = 0.01
    capacity_factor: float = 1.25
    min_expert_capacity: int = 4
    drop_overflow_tokens: bool = True
    overflow_policy: str = "drop"
    router_temperature: float = 1.0
    # ---- additions (defaults reproduce the reference architecture) ----
    norm_type: str = "layernorm"
    position_embedding: str = "learned"
    kv_heads: Optional[int] = None
    attention_bias: bool = True
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    init_std: Optional[float] = None

    def __post_init__(self) -> None:
        if self.vocab_size < 2 or self.hidden_size < 1 or self.layers < 1:
            raise ValueError("vocab_size, hidden_size, and layers must be positive")
        if self.ffn_size < 1 or self.attention_heads < 1:
            raise ValueError("ffn_size and attention_heads must be positive")
        if self.hidden_size % self.attention_heads:
            raise ValueError("hidden_size must be divisible by attention_heads")
        if self.num_experts < 1 or not 1 <= self.top_k <= self.num_experts:
            raise ValueError("top_k must be between 1 and num_experts")
        if self.max_sequence_length < 2:
            raise ValueError("max_sequence_length must be at least 2")
        if self.capacity_factor < 0 or self.min_expert_capacity < 1:
            raise ValueError("capacity_factor must be >= 0 and min_expert_capacity must be positive")
        if self.overflow_policy not in {"drop", "residual"}:
            raise ValueError("overflow_policy must be 'drop' or 'residual'")
        if self.router_temperature <= 0:
            raise ValueError("router_temperature must be positive")
        if self.norm_type not in {"layernorm", "rmsnorm"}:
            raise ValueError("norm_type must be 'layernorm' or 'rmsnorm'")
        if self.position_embedding not in {"learned", "rope"}:
            raise ValueError("position_embedding must be 'learned' or 'rope'")
        if self.kv_heads is not None:
            if self.kv_heads < 1 or self.attention_heads % self.kv_heads:
                raise ValueError("kv_heads must divide attention_heads")
        if self.position_embedding == "rope" and self.head_dim % 2:
            raise ValueError("rope needs an even head dimension")

    # ---- derived ----
    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.attention_heads

    @property
    def num_kv_heads(self) -> int:
        return self.kv_heads or self.attention_heads

    def to_dict(self) -> dict:
        return asdict(self)

    def save(self, path: Path) -> None:
        Path(path).write_text(json.dumps(self.__dict__, indent=2) + "\n")

    @classmethod
    def from_dict(cls, data: dict) -> "QuantaWeaveConfig":
        known = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in data.items() if k in known})

    @classmethod
    def load(cls, path: Path) -> "QuantaWeaveConfig":
        return cls.from_dict(json.loads(Path(path).read_text()))


# Named architectures from the benchmark configurations (tests and bench.py use these).
PRESETS: dict[str, dict] = {
    # benchmark configuration 1: CPU fp32 exact-resume gate.
    "tiny-cpu": dict(vocab_size=512, hidden_size=128, layers=4, attention_heads=4, num_experts=8, ffn_size=256,
                     top_k=2, capacity_factor=1.25, router_aux_loss_coef=0.01, norm_type="rmsnorm",
                     position_embedding="rope", attention_bias=False),
    # benchmark configuration 2: expert-parallel MoE training (the headline metric).
    "moe-1b-e64": dict(vocab_size=32000, hidden_size=1024, layers=16, attention_heads=16, num_experts=64,
                       ffn_size=2816, top_k=2, capacity_factor=1.25, router_aux_loss_coef=0.01,
                       norm_type="rmsnorm", position_embedding="rope", attention_bias=False, init_std=0.02),
    # benchmark configuration 3: Mixtral-shaped TP+EP.
    "mixtral-8x7b": dict(vocab_size=32000, hidden_size=4096, layers=32, attention_heads=32, kv_heads=8,
                         num_experts=8, ffn_size=14336, top_k=2, capacity_factor=1.0, norm_type="rmsnorm",
                         position_embedding="rope", attention_bias=False, init_std=0.02, rope_theta=1e6),
    # benchmark configuration 4: pipeline + ZeRO.
    "moe-pp-e16": dict(vocab_size=50304, hidden_size=2048, layers=24, attention_heads=16, num_experts=16,
                       ffn_size=5632, top_k=2, capacity_factor=1.25, norm_type="rmsnorm",
                       position_embedding="rope", attention_bias=False, init_std=0.02),
}


def preset(name: str, **overrides) -> QuantaWeaveConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; choose from {sorted(PRESETS)}")
    return QuantaWeaveConfig(**{**PRESETS[name], **overrides})
