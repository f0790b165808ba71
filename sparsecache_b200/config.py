"""Typed configuration: model geometry, CacheBlend, P/D and drafter settings.

Model presets cover the geometries the workloads name: the tiny CPU plumbing
decoder, Llama-3.1-8B and Llama-3.1-70B architectures (random init; no
checkpoints are downloaded), and a small head_dim-128 geometry used by the
GPU kernel tests.  Flag names mirror the reference CLIs
(src/sparsecache/qa.py:22-35, experiments/reuse_cacheblend_pipeline.py:194-236).
"""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field, replace
from typing import Any


@dataclass(frozen=True)
class RopeScaling:
    """Llama-3.1 frequency-dependent RoPE scaling ("llama3" rope type)."""

    factor: float = 8.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position_embeddings: int = 8192


@dataclass(frozen=True)
class ModelConfig:
    """Geometry of a Llama-style decoder (RMSNorm, GQA, SwiGLU, rotate-half RoPE)."""

    name: str
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rms_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: RopeScaling | None = None
    max_positions: int = 131072
    bos_token_id: int = 1
    eos_token_ids: tuple[int, ...] = ()
    # number of low ids reserved as "special" (synthetic ids avoid them)
    n_special: int = 0

    @property
    def q_size(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_rows(self) -> int:
        return self.q_size + 2 * self.kv_size

    @property
    def kv_bytes_per_token(self) -> int:
        """BF16 K+V bytes of one token over all layers."""
        return 2 * self.n_layers * self.kv_size * 2

    def n_params(self) -> int:
        per_layer = (
            self.d_model * self.qkv_rows
            + self.q_size * self.d_model
            + 3 * self.d_model * self.ffn
            + 2 * self.d_model
        )
        return self.n_layers * per_layer + 2 * self.vocab * self.d_model + self.d_model

    def to_dict(self) -> dict[str, Any]:
        data = asdict(self)
        data["eos_token_ids"] = list(self.eos_token_ids)
        return data

    def to_json(self) -> str:
        return json.dumps(self.to_dict(), sort_keys=True)

    @staticmethod
    def from_dict(data: dict[str, Any]) -> "ModelConfig":
        data = dict(data)
        scaling = data.get("rope_scaling")
        if isinstance(scaling, dict):
            data["rope_scaling"] = RopeScaling(**scaling)
        data["eos_token_ids"] = tuple(data.get("eos_token_ids", ()))
        return ModelConfig(**data)

    def with_layers(self, n_layers: int) -> "ModelConfig":
        return replace(self, n_layers=n_layers)


LLAMA3_EOS = (128001, 128008, 128009)

PRESETS: dict[str, ModelConfig] = {
    # CPU plumbing decoder: 2 layers, d 256, 4 heads / 2 KV heads, head_dim 64,
    # SwiGLU 688, RMSNorm eps 1e-5, RoPE theta 500000, vocab 1024.
    "tiny": ModelConfig(
        name="tiny",
        n_layers=2,
        d_model=256,
        n_heads=4,
        n_kv_heads=2,
        head_dim=64,
        ffn=688,
        vocab=1024,
        max_positions=8192,
        bos_token_id=1,
        eos_token_ids=(2,),
        n_special=4,
    ),
    # Small head_dim-128 geometry for GPU kernel / engine tests.
    "tiny128": ModelConfig(
        name="tiny128",
        n_layers=3,
        d_model=512,
        n_heads=4,
        n_kv_heads=2,
        head_dim=128,
        ffn=1024,
        vocab=4096,
        max_positions=16384,
        rope_scaling=RopeScaling(),
        bos_token_id=1,
        eos_token_ids=(2,),
        n_special=4,
    ),
    "llama3-8b": ModelConfig(
        name="llama3-8b",
        n_layers=32,
        d_model=4096,
        n_heads=32,
        n_kv_heads=8,
        head_dim=128,
        ffn=14336,
        vocab=128256,
        rope_scaling=RopeScaling(),
        bos_token_id=128000,
        eos_token_ids=LLAMA3_EOS,
        n_special=0,
    ),
    # Mistral-7B-Instruct-v0.2 geometry (Llama architecture, no sliding window)
    "mistral-7b": ModelConfig(
        name="mistral-7b",
        n_layers=32,
        d_model=4096,
        n_heads=32,
        n_kv_heads=8,
        head_dim=128,
        ffn=14336,
        vocab=32000,
        rope_theta=1000000.0,
        max_positions=32768,
        bos_token_id=1,
        eos_token_ids=(2,),
        n_special=3,
    ),
    "llama3-70b": ModelConfig(
        name="llama3-70b",
        n_layers=80,
        d_model=8192,
        n_heads=64,
        n_kv_heads=8,
        head_dim=128,
        ffn=28672,
        vocab=128256,
        rope_scaling=RopeScaling(),
        bos_token_id=128000,
        eos_token_ids=LLAMA3_EOS,
        n_special=0,
    ),
}


def get_model_config(name: str) -> ModelConfig:
    try:
        return PRESETS[name]
    except KeyError as exc:
        raise KeyError(f"unknown model preset {name!r}; have {sorted(PRESETS)}") from exc


DEVIATION_METRICS = ("value", "key", "kv", "value_l1", "key_l1", "kv_l1")


@dataclass(frozen=True)
class CacheBlendConfig:
    """Selective-recompute parameters (README.md:169-185 of the reference).

    ``keep_prefix`` True is the strict independent-document protocol in which
    the system prefix and the question suffix are both mandatory active rows
    (reuse_cacheblend_pipeline.py:605-616); False is the legacy
    S-conditioned path where only the suffix is mandatory (modeling.py:234-242).
    """

    check_layer: int = 1
    recompute_ratio: float = 0.15
    deviation_metric: str = "value"
    keep_prefix: bool = True
    max_new_tokens: int = 24
    # gradual filtering (the reference runner's --blend-check-layers /
    # --recompute-ratios): several ascending check layers with non-increasing
    # ratios, each relative to the ORIGINAL document token count; empty means
    # the single (check_layer, recompute_ratio)
    check_layers: tuple[int, ...] = ()
    recompute_ratios: tuple[float, ...] = ()
    # --target-average-recompute-ratio: the layer-average document fraction
    # must match within TARGET_TOLERANCE
    target_average_recompute_ratio: float | None = None

    TARGET_TOLERANCE = 0.002

    def __post_init__(self) -> None:
        if not 0 < self.recompute_ratio <= 1:
            raise ValueError("recompute_ratio must lie in (0, 1]")
        if self.deviation_metric not in DEVIATION_METRICS:
            raise ValueError(f"deviation_metric must be one of {DEVIATION_METRICS}")
        if self.check_layer < 0:
            raise ValueError("check_layer must be non-negative")
        if self.check_layers or self.recompute_ratios:
            layers, ratios = tuple(self.check_layers), tuple(self.recompute_ratios)
            if len(layers) != len(ratios) or not layers:
                raise ValueError("check_layers and recompute_ratios must have the same non-zero length")
            if any(b <= a for a, b in zip(layers, layers[1:])) or layers[0] < 0:
                raise ValueError("check_layers must be ascending and non-negative")
            if any(not 0 < r <= 1 for r in ratios) or any(b > a for a, b in zip(ratios, ratios[1:])):
                raise ValueError("recompute_ratios must lie in (0, 1] and not increase")
            object.__setattr__(self, "check_layers", layers)
            object.__setattr__(self, "recompute_ratios", ratios)
            object.__setattr__(self, "check_layer", layers[0])
            object.__setattr__(self, "recompute_ratio", ratios[-1])

    @property
    def schedule(self) -> tuple[tuple[int, float], ...]:
        """(check layer, retained document ratio) pairs in layer order."""
        if self.check_layers:
            return tuple(zip(self.check_layers, self.recompute_ratios))
        return ((self.check_layer, self.recompute_ratio),)

    def layer_document_trace(self, n_layers: int) -> list[float]:
        """Fraction of the document tokens each layer processes (1.0 up to the first check layer)."""
        sched = self.schedule
        if sched[-1][0] >= n_layers:
            raise ValueError("a check layer lies outside the model")
        trace, frac = [], 1.0
        for layer in range(n_layers):
            trace.append(frac)
            for c, r in sched:
                if c == layer:
                    frac = r
        return trace

    def check_target(self, n_layers: int) -> float:
        """Mean of the layer trace; raises if a target average is set and missed by > 0.002."""
        trace = self.layer_document_trace(n_layers)
        mean = sum(trace) / len(trace)
        t = self.target_average_recompute_ratio
        if t is not None and abs(mean - t) > self.TARGET_TOLERANCE:
            raise ValueError(f"layer-average document ratio {mean:.6f} misses the target {t} by more than "
                             f"{self.TARGET_TOLERANCE}")
        return mean

    @property
    def dev_mode(self) -> int:
        """Bit mask understood by the fused deviation epilogue (1 key, 2 value, 4 L1)."""
        metric = self.deviation_metric
        mode = 0
        if metric.startswith("key") or metric.startswith("kv"):
            mode |= 1
        if metric.startswith("value") or metric.startswith("kv"):
            mode |= 2
        if metric.endswith("_l1"):
            mode |= 4
        return mode


@dataclass(frozen=True)
class ProgressiveConfig:
    """Progressive P/D transfer and drafting parameters (pd_progressive_kv_pipeline.py:459-616)."""

    stage_fractions: tuple[float, ...] = (0.1, 0.4, 0.7, 1.0)
    anchor_tokens: int = 256
    draft_tokens: int = 4
    commit_window: int | None = None  # None = W infinity (single final verifier)
    transport_gbps: float | None = None
    eager_serial_wire: bool = False
    page_tokens: int = 64


@dataclass(frozen=True)
class DrafterConfig:
    """Sparse-KV drafter geometry and memory selection."""

    hidden: int = 512
    heads: int = 4
    head_dim: int = 128
    memory_heads: int = 8
    memory_layers: tuple[int, ...] = (8, 20, 31)
    seed_layers: tuple[int, ...] = (2, 16, 29)
    sink_tokens: int = 64
    recent_tokens: int = 512
    chunk_tokens: int = 64
    chunk_budget: int = 2048
    extra: dict[str, Any] = field(default_factory=dict)
