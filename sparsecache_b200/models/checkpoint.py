"""Model directories: ``config.json`` + ``model.safetensors`` (+ index).

Parameter names follow the usual Llama naming (``model.layers.N.self_attn.q_proj.weight``
...) so the directory is self-describing; ``model_fingerprint`` of the store
hashes ``config.json`` and ``model.safetensors.index.json`` exactly as the
reference does for HF checkpoints (store.py:19-27).

Hugging Face Llama / Mistral directories load as they are: a ``config.json``
with ``num_hidden_layers`` is read as an HF config (GQA head counts,
``head_dim``, ``rope_theta``, the "llama3" ``rope_scaling`` block, EOS ids,
tied embeddings), and weights come from ``model.safetensors`` or from the
shards named by ``model.safetensors.index.json``.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import torch
from safetensors.torch import load_file, save_file

from ..config import ModelConfig, RopeScaling, get_model_config
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


def config_from_hf(data: dict, name: str = "hf") -> ModelConfig:
    """ModelConfig of a Hugging Face Llama-family ``config.json``."""
    arch = set(data.get("architectures") or ())
    if arch and not arch & {"LlamaForCausalLM", "MistralForCausalLM"}:
        raise ValueError(f"unsupported architecture {sorted(arch)}: the engine implements the Llama geometry")
    if data.get("sliding_window") not in (None, 0) and int(data["sliding_window"]) < int(
            data.get("max_position_embeddings", 0)):
        raise ValueError("sliding-window attention is not implemented")
    heads = int(data["num_attention_heads"])
    # transformers < 5 writes rope_theta + rope_scaling; >= 5 one rope_parameters block
    params = data.get("rope_parameters") or {}
    scaling = data.get("rope_scaling") or params
    theta = float(data.get("rope_theta") or params.get("rope_theta") or 10000.0)
    rope = None
    kind = scaling.get("rope_type", scaling.get("type")) if scaling else None
    if kind not in (None, "default"):
        if kind != "llama3":
            raise ValueError(f"unsupported rope scaling {kind!r}")
        rope = RopeScaling(factor=float(scaling["factor"]), low_freq_factor=float(scaling["low_freq_factor"]),
                           high_freq_factor=float(scaling["high_freq_factor"]),
                           original_max_position_embeddings=int(scaling["original_max_position_embeddings"]))
    eos = data.get("eos_token_id")
    eos_ids = () if eos is None else ((int(eos),) if isinstance(eos, int) else tuple(int(x) for x in eos))
    return ModelConfig(name=name, n_layers=int(data["num_hidden_layers"]), d_model=int(data["hidden_size"]),
                       n_heads=heads, n_kv_heads=int(data.get("num_key_value_heads", heads)),
                       head_dim=int(data.get("head_dim") or int(data["hidden_size"]) // heads),
                       ffn=int(data["intermediate_size"]), vocab=int(data["vocab_size"]),
                       rms_eps=float(data.get("rms_norm_eps", 1e-5)), rope_theta=theta,
                       rope_scaling=rope, max_positions=int(data.get("max_position_embeddings", 131072)),
                       bos_token_id=int(data.get("bos_token_id", 1) or 1), eos_token_ids=eos_ids)


def load_config(directory: str | Path) -> ModelConfig:
    data = json.loads((Path(directory) / "config.json").read_text(encoding="utf-8"))
    if "num_hidden_layers" in data:
        return config_from_hf(data, name=Path(directory).name)
    return ModelConfig.from_dict(data)


def _weights(directory: Path) -> dict[str, torch.Tensor]:
    single = directory / "model.safetensors"
    index = directory / "model.safetensors.index.json"
    if index.exists():
        shards = sorted(set(json.loads(index.read_text(encoding="utf-8"))["weight_map"].values()))
        out: dict[str, torch.Tensor] = {}
        for shard in shards:
            out.update(load_file(str(directory / shard), device="cpu"))
        return out
    return load_file(str(single), device="cpu")


def load_oracle(directory: str | Path, *, dtype: torch.dtype = torch.float32, device="cpu") -> LlamaOracle:
    directory = Path(directory)
    cfg = load_config(directory)
    model = LlamaOracle(cfg)
    tensors = _weights(directory)
    if "lm_head.weight" not in tensors:  # tied embeddings
        tensors["lm_head.weight"] = tensors["model.embed_tokens.weight"]
    params = dict(model.named_parameters())
    missing = [n for n, _ in _names(cfg) if n not in tensors]
    if missing:
        raise ValueError(f"checkpoint lacks {len(missing)} tensors, e.g. {missing[:3]}")
    with torch.no_grad():
        for name, (module, attr) in _names(cfg):
            t = tensors[name]
            if tuple(t.shape) != tuple(params[f"{module}.{attr}"].shape):
                raise ValueError(f"{name}: shape {tuple(t.shape)} differs from the config's")
            params[f"{module}.{attr}"].copy_(t)
    return model.to(device=device, dtype=dtype).eval()


def random_checkpoint(directory: str | Path, preset: str, *, seed: int = 0, std: float = 0.02) -> Path:
    """Write a seeded random-init model directory for ``preset`` (no download)."""
    model = LlamaOracle.random_init(get_model_config(preset), seed=seed, std=std)
    return save_checkpoint(directory, model)


def checkpoint_shard(directory: str | Path, rank: int, tp: int, device="cpu"):
    """Engine weights of tensor-parallel ``rank`` read straight from a model directory.

    Only this rank's rows / columns are read from the safetensors files
    (column-parallel q/k/v heads and gate/up rows, row-parallel o / down
    columns; norms, embedding and LM head replicated), so a 70B checkpoint
    never has to fit one host whole.  The result equals slicing the full
    engine weights with ``parallel.tp.shard_weights``.
    """
    from safetensors import safe_open

    from .engine import EngineWeights, LayerWeights
    from .weights import GATE_UP_BLOCK, fuse_qkv, interleave_gate_up

    directory = Path(directory)
    cfg = load_config(directory)
    if cfg.n_heads % tp or cfg.n_kv_heads % tp or cfg.ffn % (tp * GATE_UP_BLOCK):
        raise ValueError("heads, kv heads and ffn / 128 must divide by the TP size")
    index = directory / "model.safetensors.index.json"
    where = (json.loads(index.read_text(encoding="utf-8"))["weight_map"] if index.exists() else None)
    handles: dict[str, Any] = {}

    def sl(name: str):
        if where is not None and name not in where:
            raise KeyError(name)
        fname = where[name] if where is not None else "model.safetensors"
        if fname not in handles:
            handles[fname] = safe_open(str(directory / fname), framework="pt", device="cpu")
        if name not in handles[fname].keys():
            raise KeyError(name)
        return handles[fname].get_slice(name)

    bf = torch.bfloat16
    dev = torch.device(device)

    def t(x):
        return x.to(device=dev, dtype=bf).contiguous()

    D = cfg.head_dim
    hq, hkv, f = cfg.n_heads // tp, cfg.n_kv_heads // tp, cfg.ffn // tp
    layers = []
    for i in range(cfg.n_layers):
        b = f"model.layers.{i}."
        q = sl(b + "self_attn.q_proj.weight")[rank * hq * D:(rank + 1) * hq * D]
        k = sl(b + "self_attn.k_proj.weight")[rank * hkv * D:(rank + 1) * hkv * D]
        v = sl(b + "self_attn.v_proj.weight")[rank * hkv * D:(rank + 1) * hkv * D]
        gate = sl(b + "mlp.gate_proj.weight")[rank * f:(rank + 1) * f]
        up = sl(b + "mlp.up_proj.weight")[rank * f:(rank + 1) * f]
        layers.append(LayerWeights(
            ln1=t(sl(b + "input_layernorm.weight")[:]), w_qkv=t(fuse_qkv(q, k, v)),
            w_o=t(sl(b + "self_attn.o_proj.weight")[:, rank * hq * D:(rank + 1) * hq * D]),
            ln2=t(sl(b + "post_attention_layernorm.weight")[:]), w_gu=t(interleave_gate_up(gate, up)),
            w_down=t(sl(b + "mlp.down_proj.weight")[:, rank * f:(rank + 1) * f])))
    embed = t(sl("model.embed_tokens.weight")[:])
    try:
        head = t(sl("lm_head.weight")[:])
    except KeyError:  # tied embeddings
        head = embed
    return cfg, EngineWeights(embed=embed, layers=layers, norm=t(sl("model.norm.weight")[:]), lm_head=head)
