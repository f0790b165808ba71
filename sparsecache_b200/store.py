"""Portable BF16 KV files, manifests, and the deduplicating document KV store.

On-disk format (kept identical to the reference so caches interoperate,
src/sparsecache/store.py:39-96):
  * one safetensors file per cached segment with tensors
    ``layer_{i:03d}.key`` / ``layer_{i:03d}.value`` of shape
    [1, n_kv_heads, tokens, head_dim], written atomically (.tmp + rename);
  * ``manifest.json`` with ``format == "sparsecache.chunk-kv.v1"``;
  * the model fingerprint is the sha256 of config.json and
    model.safetensors.index.json (for random-init models: of the config JSON,
    the seed and the weight shapes).

In memory, the B200 store keeps each unique document as ONE contiguous
[L, 2, n_kv_heads, tokens, head_dim] bf16 block, either resident in HBM
(180 GB per B200 holds tens of thousands of documents next to an 8B model)
or in pinned host memory that the composer kernel reads directly over PCIe.
Documents are deduplicated by their exact token-id tuple
(reuse_cacheblend_pipeline.py:354-386).
"""
from __future__ import annotations

import hashlib
import json
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Iterable, Sequence

import torch
from safetensors.torch import load_file, save_file

from .config import ModelConfig
from .rope import relocate_key

LegacyCache = tuple[tuple[torch.Tensor, torch.Tensor], ...]
MANIFEST_FORMAT = "sparsecache.chunk-kv.v1"


# ------------------------------------------------------------- fingerprints
def model_fingerprint(model_path: str | Path) -> str:
    """sha256 over config.json and model.safetensors.index.json (when present)."""
    root = Path(model_path)
    digest = hashlib.sha256()
    for name in ("config.json", "model.safetensors.index.json"):
        path = root / name
        if path.exists():
            digest.update(path.read_bytes())
    return digest.hexdigest()


def config_fingerprint(config: ModelConfig, seed: int) -> str:
    """Fingerprint of a random-init model: config JSON, seed and weight-shape index."""
    digest = hashlib.sha256()
    digest.update(config.to_json().encode())
    digest.update(f"seed={seed}".encode())
    shapes = {
        "embed": [config.vocab, config.d_model],
        "qkv": [config.qkv_rows, config.d_model],
        "o": [config.d_model, config.q_size],
        "gate_up": [2 * config.ffn, config.d_model],
        "down": [config.d_model, config.ffn],
        "lm_head": [config.vocab, config.d_model],
    }
    digest.update(json.dumps(shapes, sort_keys=True).encode())
    return digest.hexdigest()


# --------------------------------------------------------------- file format
def cache_to_legacy(cache: Any) -> LegacyCache:
    """Normalise a cache object into per-layer (key, value) tuples."""
    if hasattr(cache, "to_legacy_cache"):
        return tuple(cache.to_legacy_cache())
    if isinstance(cache, (tuple, list)):
        return tuple((k, v) for k, v in cache)
    raise TypeError(f"unsupported cache object: {type(cache)!r}")


def save_cache(path: str | Path, cache: LegacyCache) -> int:
    """Write a cache as safetensors (atomic); returns the logical K+V byte count."""
    tensors = {}
    logical = 0
    for index, (key, value) in enumerate(cache):
        key = key.detach().to("cpu").contiguous()
        value = value.detach().to("cpu").contiguous()
        tensors[f"layer_{index:03d}.key"] = key
        tensors[f"layer_{index:03d}.value"] = value
        logical += (key.numel() + value.numel()) * key.element_size()
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    save_file(tensors, str(tmp))
    tmp.replace(path)
    return logical


def load_cache(path: str | Path, expected_layers: int | None = None) -> LegacyCache:
    """Read a safetensors cache into CPU tensors, layers in index order."""
    tensors = load_file(str(path), device="cpu")
    layers = sorted(int(name.split(".")[0].split("_")[1]) for name in tensors if name.endswith(".key"))
    if expected_layers is not None and len(layers) != expected_layers:
        raise ValueError(f"cache has {len(layers)} layers, expected {expected_layers}")
    return tuple((tensors[f"layer_{i:03d}.key"], tensors[f"layer_{i:03d}.value"]) for i in layers)


def slice_cache(cache: Any, start: int, end: int) -> LegacyCache:
    """CPU copy of the token interval [start, end) of every layer."""
    return tuple(
        (k[:, :, start:end].detach().to("cpu").contiguous(), v[:, :, start:end].detach().to("cpu").contiguous())
        for k, v in cache_to_legacy(cache)
    )


def cache_bytes(cache: LegacyCache) -> int:
    return sum((k.numel() + v.numel()) * k.element_size() for k, v in cache)


def load_manifest(path: str | Path) -> dict[str, Any]:
    manifest_path = Path(path)
    manifest = json.loads(manifest_path.read_text(encoding="utf-8"))
    if manifest.get("format") != MANIFEST_FORMAT:
        raise ValueError("unsupported SparseCache manifest format")
    manifest["_root"] = str(manifest_path.parent.resolve())
    return manifest


@torch.inference_mode()
def compose_cache(config: ModelConfig, manifest: dict[str, Any]) -> tuple[LegacyCache, dict[str, Any]]:
    """Load the system and chunk caches of a manifest, relocate chunk keys, concatenate.

    Reference: store.py:99-149 (there the RoPE schedule comes from the HF
    model; here from the model config).
    """
    root = Path(manifest["_root"])
    layers = int(manifest["model"]["layers"])
    system = load_cache(root / manifest["system"]["file"], layers)
    keys = [[k] for k, _ in system]
    values = [[v] for _, v in system]
    cursor = int(manifest["system"]["tokens"])
    ranges = []
    relocated = 0
    for chunk in manifest["chunks"]:
        chunk_cache = load_cache(root / chunk["file"], layers)
        source_start = int(chunk["source_start"])
        tokens = int(chunk["tokens"])
        for index, (key, value) in enumerate(chunk_cache):
            keys[index].append(relocate_key(config, key, source_start=source_start, target_start=cursor))
            values[index].append(value)
        if source_start != cursor:
            relocated += tokens
        ranges.append({"chunk_id": chunk["chunk_id"], "title": chunk.get("title", ""), "start": cursor, "end": cursor + tokens})
        cursor += tokens
    composed = tuple((torch.cat(keys[i], dim=2), torch.cat(values[i], dim=2)) for i in range(layers))
    system_tokens = int(manifest["system"]["tokens"])
    return composed, {
        "system_tokens": system_tokens,
        "document_tokens": cursor - system_tokens,
        "prefix_tokens": cursor,
        "relocated_tokens": relocated,
        "chunk_ranges": ranges,
    }


# ------------------------------------------------------- document KV store
@dataclass
class DocumentEntry:
    """One unique document: token ids and its K/V block [L, 2, Hkv, n, D]."""

    tokens: tuple[int, ...]
    kv: torch.Tensor

    @property
    def n_tokens(self) -> int:
        return len(self.tokens)

    def legacy(self) -> LegacyCache:
        return tuple((self.kv[i, 0].unsqueeze(0), self.kv[i, 1].unsqueeze(0)) for i in range(self.kv.shape[0]))

    def nbytes(self) -> int:
        return self.kv.numel() * self.kv.element_size()


def stack_legacy(cache: LegacyCache) -> torch.Tensor:
    """[(k [1,H,n,D], v)] * L  ->  [L, 2, H, n, D]."""
    return torch.stack([torch.stack((k[0], v[0])) for k, v in cache])


class DocumentKVStore:
    """Deduplicated per-document KV keyed by exact token sequence.

    ``tier`` is where the blocks live: "hbm" (device-resident, the default on
    a B200) or "pinned" (page-locked host memory, read by the composer kernel
    over PCIe) or "cpu" (pageable, oracle path).
    """

    def __init__(self, config: ModelConfig, *, tier: str = "hbm", device: torch.device | str | None = None) -> None:
        if tier not in ("hbm", "pinned", "cpu"):
            raise ValueError("tier must be hbm, pinned or cpu")
        self.config = config
        self.tier = tier
        self.device = torch.device(device) if device is not None else None
        self.entries: dict[tuple[int, ...], DocumentEntry] = {}
        self.stats: dict[str, Any] = {"unique_documents": 0, "producer_calls": 0, "logical_bytes": 0, "wall_ms": 0.0}

    def __contains__(self, tokens: Sequence[int]) -> bool:
        return tuple(tokens) in self.entries

    def __getitem__(self, tokens: Sequence[int]) -> DocumentEntry:
        return self.entries[tuple(tokens)]

    def __len__(self) -> int:
        return len(self.entries)

    def _place(self, kv: torch.Tensor) -> torch.Tensor:
        if self.tier == "hbm":
            return kv.to(self.device or kv.device).contiguous()
        if self.tier == "pinned":
            out = torch.empty(kv.shape, dtype=kv.dtype, pin_memory=True)
            out.copy_(kv)
            return out
        return kv.to("cpu").contiguous()

    def put(self, tokens: Sequence[int], kv: torch.Tensor) -> DocumentEntry:
        key = tuple(int(t) for t in tokens)
        entry = DocumentEntry(key, self._place(kv))
        self.entries[key] = entry
        self.stats["unique_documents"] = len(self.entries)
        self.stats["logical_bytes"] += entry.nbytes()
        return entry

    def produce(self, producer, documents: Iterable[Sequence[int]]) -> dict[str, Any]:
        """Prefill every not-yet-stored document alone at local positions 0..n-1.

        ``producer(tokens) -> [L, 2, Hkv, n, D]`` (the engine's or the oracle's
        local encoder).  Returns producer statistics (unique_documents,
        producer_calls, logical_bytes, wall_ms), as the reference reports.
        """
        started = time.perf_counter()
        calls = 0
        for tokens in documents:
            key = tuple(int(t) for t in tokens)
            if key in self.entries:
                continue
            self.put(key, producer(key))
            calls += 1
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self.stats["producer_calls"] += calls
        self.stats["wall_ms"] += (time.perf_counter() - started) * 1000
        return dict(self.stats)

    def total_bytes(self) -> int:
        return sum(e.nbytes() for e in self.entries.values())

    # --------------------------------------------------------- persistence
    def save(self, directory: str | Path, fingerprint: str) -> Path:
        """One safetensors file per document (reference tensor layout) + index."""
        root = Path(directory)
        root.mkdir(parents=True, exist_ok=True)
        index = []
        for tokens, entry in self.entries.items():
            name = hashlib.sha256(json.dumps(tokens).encode()).hexdigest()[:32] + ".safetensors"
            save_cache(root / name, entry.legacy())
            index.append({"file": name, "tokens": list(tokens)})
        meta = {"format": "sparsecache.document-kv-store.v1", "fingerprint": fingerprint,
                "model": self.config.to_dict(), "documents": index}
        tmp = root / "store.json.tmp"
        tmp.write_text(json.dumps(meta), encoding="utf-8")
        tmp.replace(root / "store.json")
        return root / "store.json"

    @classmethod
    def load(cls, directory: str | Path, config: ModelConfig, fingerprint: str, **kw) -> "DocumentKVStore":
        root = Path(directory)
        meta = json.loads((root / "store.json").read_text(encoding="utf-8"))
        if meta.get("format") != "sparsecache.document-kv-store.v1":
            raise ValueError("unsupported document store format")
        if meta.get("fingerprint") != fingerprint:
            raise ValueError("document store was produced by a different model")
        store = cls(config, **kw)
        for item in meta["documents"]:
            store.put(item["tokens"], stack_legacy(load_cache(root / item["file"], config.n_layers)))
        return store
