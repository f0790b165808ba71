"""Model directories: ``config.json`` + ``model.safetensors`` (+ index).

Parameter names follow the usual Llama naming (``model.layers.N.self_attn.q_proj.weight``
...) so the directory is self-describing; ``model_fingerprint`` of the store
hashes ``config.json`` and ``model.safetensors.index.json`` exactly as the
reference does for HF checkpoints (store.py:19-27).
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
from safetensors.torch import load_file, save_file

from ..config import ModelConfig, get_model_config
from .llama import LlamaOracle


def _names(cfg: ModelConfig):
    yield "model.embed_tokens.weight", ("embed_tokens", "weight")
    for i in range(cfg.n_layers):
        base = f"model.layers.{i}."
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
            yield base + f"self_attn.{proj}.weight", (f"layers.{i}.{proj}", "weight")
        for proj in ("gate_proj", "up_proj", "down_proj"):
            yield base + f"mlp.{proj}.weight", (f"layers.{i}.{proj}", "weight")
        yield base + "input_layernorm.weight", (f"layers.{i}.input_layernorm", "weight")
        yield base + "post_attention_layernorm.weight", (f"layers.{i}.post_attention_layernorm", "weight")
    yield "model.norm.weight", ("norm", "weight")
    yield "lm_head.weight", ("lm_head", "weight")


def save_checkpoint(directory: str | Path, model: LlamaOracle, *, dtype: torch.dtype = torch.bfloat16) -> Path:
    root = Path(directory)
    root.mkdir(parents=True, exist_ok=True)
    params = dict(model.named_parameters())
    tensors = {}
    for name, (module, attr) in _names(model.config):
        tensors[name] = params[f"{module}.{attr}"].detach().to("cpu", dtype).contiguous()
    save_file(tensors, str(root / "model.safetensors"))
    index = {"metadata": {"total_size": sum(t.numel() * t.element_size() for t in tensors.values())},
             "weight_map": {k: "model.safetensors" for k in sorted(tensors)}}
    (root / "model.safetensors.index.json").write_text(json.dumps(index, indent=1), encoding="utf-8")
    (root / "config.json").write_text(json.dumps(model.config.to_dict(), indent=1, sort_keys=True), encoding="utf-8")
    return root


def load_config(directory: str | Path) -> ModelConfig:
    return ModelConfig.from_dict(json.loads((Path(directory) / "config.json").read_text(encoding="utf-8")))


def load_oracle(directory: str | Path, *, dtype: torch.dtype = torch.float32, device="cpu") -> LlamaOracle:
    cfg = load_config(directory)
    model = LlamaOracle(cfg)
    tensors = load_file(str(Path(directory) / "model.safetensors"), device="cpu")
    params = dict(model.named_parameters())
    with torch.no_grad():
        for name, (module, attr) in _names(cfg):
            params[f"{module}.{attr}"].copy_(tensors[name])
    return model.to(device=device, dtype=dtype).eval()


def random_checkpoint(directory: str | Path, preset: str, *, seed: int = 0, std: float = 0.02) -> Path:
    """Write a seeded random-init model directory for ``preset`` (no download)."""
    model = LlamaOracle.random_init(get_model_config(preset), seed=seed, std=std)
    return save_checkpoint(directory, model)
