"""Model architecture configs and presets.

The reference resolves architectures through HF ``AutoConfig`` and a registry
(python/lake/engine/model_executor/models/registry.py:52-124). Here a config can
come from a preset name, an HF ``config.json`` (``from_hf_dict``) or keyword
overrides; weights are random-initialised (no checkpoints on this box).
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field


@dataclass
class ModelConfig:
    name: str = "llama3-8b"
    arch: str = "llama"  # llama | mixtral | qwen3
    hidden: int = 4096
    n_layers: int = 32
    n_q_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None
    rms_eps: float = 1e-5
    tie_embeddings: bool = False
    n_experts: int = 0
    top_k: int = 0
    qk_norm: bool = False
    max_position: int = 8192
    dtype: str = "bfloat16"
    extra: dict = field(default_factory=dict)

    @property
    def q_size(self) -> int:
        return self.n_q_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def group(self) -> int:
        return self.n_q_heads // self.n_kv_heads

    def kv_bytes_per_token(self, elem_bytes: int = 2) -> int:
        return self.n_layers * 2 * self.kv_size * elem_bytes

    def num_params(self) -> int:
        h, i, L = self.hidden, self.intermediate, self.n_layers
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        mlp = 3 * h * i * max(1, self.n_experts) + (h * self.n_experts if self.n_experts else 0)
        emb = self.vocab * h * (1 if self.tie_embeddings else 2)
        return L * (attn + mlp + 2 * h) + emb + h

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    @staticmethod
    def from_hf_dict(d: dict, name: str = "hf") -> "ModelConfig":
        """Map an HF config.json dict (LlamaForCausalLM / MixtralForCausalLM / Qwen3ForCausalLM)."""
        archs = d.get("architectures") or []
        arch = "llama"
        if any("Mixtral" in a for a in archs) or d.get("num_local_experts"):
            arch = "mixtral"
        elif any("Qwen3" in a for a in archs):
            arch = "qwen3"
        hq = d["num_attention_heads"]
        return ModelConfig(
            name=name, arch=arch, hidden=d["hidden_size"], n_layers=d["num_hidden_layers"], n_q_heads=hq,
            n_kv_heads=d.get("num_key_value_heads", hq), head_dim=d.get("head_dim") or d["hidden_size"] // hq,
            intermediate=d["intermediate_size"], vocab=d["vocab_size"], rope_theta=float(d.get("rope_theta", 1e4)),
            rope_scaling=d.get("rope_scaling"), rms_eps=float(d.get("rms_norm_eps", 1e-5)),
            tie_embeddings=bool(d.get("tie_word_embeddings", False)), n_experts=int(d.get("num_local_experts", 0)),
            top_k=int(d.get("num_experts_per_tok", 0)), qk_norm=arch == "qwen3",
            max_position=int(d.get("max_position_embeddings", 8192)))

    @staticmethod
    def from_json(path: str) -> "ModelConfig":
        with open(path) as f:
            d = json.load(f)
        if "hidden_size" in d:
            return ModelConfig.from_hf_dict(d, name=os.path.basename(os.path.dirname(path)) or "hf")
        return ModelConfig(**d)


PRESETS: dict[str, ModelConfig] = {
    # 2-layer plumbing model (CPU, fp32): hidden 256, 4 q / 2 kv heads, head_dim 64, FFN 1024, vocab 1024.
    "tiny": ModelConfig(name="tiny", hidden=256, n_layers=2, n_q_heads=4, n_kv_heads=2, head_dim=64,
                        intermediate=1024, vocab=1024, rope_theta=10000.0, max_position=4096, dtype="float32"),
    # Small GPU test model that satisfies the kernels' constraints (head_dim 128).
    "tiny-gpu": ModelConfig(name="tiny-gpu", hidden=512, n_layers=2, n_q_heads=4, n_kv_heads=2, head_dim=128,
                            intermediate=1024, vocab=2048, rope_theta=10000.0, max_position=8192),
    "llama3-8b": ModelConfig(name="llama3-8b"),
    "llama3-70b": ModelConfig(name="llama3-70b", hidden=8192, n_layers=80, n_q_heads=64, n_kv_heads=8,
                              intermediate=28672),
    "mixtral-8x7b": ModelConfig(name="mixtral-8x7b", arch="mixtral", hidden=4096, n_layers=32, n_q_heads=32,
                                n_kv_heads=8, intermediate=14336, vocab=32000, rope_theta=1e6, n_experts=8,
                                top_k=2, max_position=32768),
    "qwen3-0.6b": ModelConfig(name="qwen3-0.6b", arch="qwen3", hidden=1024, n_layers=28, n_q_heads=16,
                              n_kv_heads=8, head_dim=128, intermediate=3072, vocab=151936, rope_theta=1e6,
                              rms_eps=1e-6, tie_embeddings=True, qk_norm=True, max_position=40960),
}


def get_config(name_or_path: str, **overrides) -> ModelConfig:
    if name_or_path in PRESETS:
        cfg = PRESETS[name_or_path]
    elif os.path.isdir(name_or_path) and os.path.exists(os.path.join(name_or_path, "config.json")):
        cfg = ModelConfig.from_json(os.path.join(name_or_path, "config.json"))
    elif os.path.isfile(name_or_path):
        cfg = ModelConfig.from_json(name_or_path)
    else:
        raise KeyError(f"unknown model {name_or_path!r}; presets: {sorted(PRESETS)}")
    return cfg.replace(**overrides) if overrides else cfg
