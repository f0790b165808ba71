"""Document KV on disk, streamed into HBM layer by layer while CacheBlend runs.

The reference's CacheBlend setup can keep the per-document KV on SSD and load
it per layer through two pinned buffers with a CUDA event per layer, in a
"disk_sync" (load everything, then compute) and a "disk_async" (compute on
layer l while later layers load) mode (README.md:254-282; about 745 MB per
request over 31 layers, README.md:285-287).  Here:

  * ``DiskKVStore`` writes each unique document once in the reference's
    chunk-KV format (safetensors, tensors ``layer_NNN.key`` / ``layer_NNN.value``
    of shape [1, kv_heads, tokens, head_dim], atomic ``.tmp`` + rename,
    ``sparsecache.store.save_cache``), keyed by the exact token sequence;
  * ``safetensors_extents`` reads a file's header (little-endian u64 length +
    JSON) into byte extents, so no tensor data is parsed in Python;
  * ``LayerwiseDiskKV`` hands the per-layer extents of a request's documents
    to the native loader (``LayerwiseKVLoader`` in ops/csrc/disk_loader.cpp:
    pread workers -> pinned double buffer -> H2D on its own stream -> a ready
    event per layer) with one HBM block [L, 2, H_kv, n, D] per document as
    the destination;
  * ``blend_from_disk`` runs ``B200Engine.cacheblend`` with a per-layer hook
    that waits for the layer's event on the compute stream and composes that
    layer only, so reading layer l+1.. overlaps the recompute of layer l.
"""
from __future__ import annotations

import hashlib
import json
import struct
from pathlib import Path
from typing import Sequence

import torch

from ..store import save_cache


def safetensors_extents(path: str | Path) -> dict[str, tuple[int, int, tuple[int, ...], str]]:
    """name -> (byte offset in the file, byte count, shape, dtype) from the safetensors header."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    base = 8 + n
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        b, e = meta["data_offsets"]
        out[name] = (base + b, e - b, tuple(meta["shape"]), meta["dtype"])
    return out


def document_key(tokens: Sequence[int]) -> str:
    return hashlib.sha256(json.dumps([int(t) for t in tokens]).encode()).hexdigest()[:32]


class DiskKVStore:
    """One safetensors chunk-KV file per unique document under ``root``."""

    def __init__(self, root: str | Path, config) -> None:
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)
        self.config = config

    def path(self, tokens: Sequence[int]) -> Path:
        return self.root / f"{document_key(tokens)}.safetensors"

    def __contains__(self, tokens) -> bool:
        return self.path(tokens).exists()

    def put(self, tokens: Sequence[int], block: torch.Tensor) -> Path:
        """Write a [L, 2, H_kv, n, D] block in the chunk-KV layout (no-op if present)."""
        p = self.path(tokens)
        if not p.exists():
            L = block.shape[0]
            save_cache(p, tuple((block[l, 0].unsqueeze(0), block[l, 1].unsqueeze(0)) for l in range(L)))
        return p

    def put_all(self, memory_store) -> int:
        """Write every document of an in-memory ``DocumentKVStore``; returns files written."""
        n = 0
        for tokens, entry in memory_store.entries.items():
            if tokens not in self:
                self.put(tokens, entry.kv)
                n += 1
        return n


class LayerwiseDiskKV:
    """Per-request layer-wise loader: document files -> one HBM block per document."""

    def __init__(self, config, device, *, staging_bytes: int = 64 << 20, n_buffers: int = 2, n_threads: int = 4,
                 host: bool = False) -> None:
        self.cfg = config
        self.device = torch.device(device) if not host else torch.device("cpu")
        self.host = host
        self.staging_bytes = int(staging_bytes)
        self.n_buffers, self.n_threads = n_buffers, n_threads
        self._loader = None
        self._buf: torch.Tensor | None = None

    def start(self, paths: Sequence[str | Path], layers: Sequence[int]) -> list[torch.Tensor]:
        """Start streaming ``layers`` (ascending) of every file; returns the destination blocks.

        Block i is [L, 2, H_kv, n_i, D] bf16; only the streamed layers are
        written.  Layer ``layers[j]`` is ready after ``wait_layer(layers[j])``.
        """
        from .. import ops

        cfg = self.cfg
        L, H, D = cfg.n_layers, cfg.n_kv_heads, cfg.head_dim
        metas = [safetensors_extents(p) for p in paths]
        ns = []
        for p, m in zip(paths, metas):
            shape = m["layer_000.key"][2]
            if len(shape) != 4 or shape[1] != H or shape[3] != D or sum(k.endswith(".key") for k in m) != L:
                raise ValueError(f"{p}: not a [1, {H}, n, {D}] x {L}-layer chunk-KV file")
            ns.append(shape[2])
        total = sum(L * 2 * H * n * D for n in ns)
        dev = self.device
        if self._buf is None or self._buf.numel() < total:
            self._buf = torch.empty(total, dtype=torch.bfloat16, device=dev)
        blocks, base = [], 0
        for n in ns:
            blocks.append(self._buf[base:base + L * 2 * H * n * D].view(L, 2, H, n, D))
            base += L * 2 * H * n * D
        self.layers = list(layers)
        self._index = {l: j for j, l in enumerate(self.layers)}
        plan = []
        for l in self.layers:
            rows = []
            for i, (m, blk) in enumerate(zip(metas, blocks)):
                for kind, name in ((0, f"layer_{l:03d}.key"), (1, f"layer_{l:03d}.value")):
                    off, nb, _, dtype = m[name]
                    if dtype != "BF16":
                        raise ValueError("chunk-KV files must be bf16")
                    dst = blk[l, kind]
                    rows.append([i, off, nb, dst.data_ptr() - self._buf.data_ptr()])
            plan.append(rows)
        need = max((sum(r[2] for r in rows) for rows in plan), default=0)
        if self._loader is None or need > self.staging_bytes:
            if self._loader is not None:
                self._loader.join()
            self.staging_bytes = max(self.staging_bytes, need)
            self._loader = ops.ext().LayerwiseKVLoader(self.staging_bytes, self.n_buffers, self.n_threads,
                                                       -1 if self.host else dev.index)
        after = 0 if self.host else torch.cuda.current_stream(dev).cuda_stream
        self._loader.start([str(p) for p in paths], plan, self._buf.data_ptr(), after)
        return blocks

    def wait_layer(self, layer: int, stream: torch.cuda.Stream | None = None) -> None:
        s = 0
        if not self.host:
            s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        self._loader.wait_layer(self._index[layer], s)

    def join(self) -> dict:
        self._loader.join()
        return dict(self._loader.stats())


def blend_from_disk(engine, slot, request, ids: torch.Tensor, disk: DiskKVStore, loader: LayerwiseDiskKV, *,
                    blend, mode: str = "async"):
    """CacheBlend whose document KV comes from disk, composed layer by layer.

    ``mode`` "async" overlaps reading layer l+1.. with the recompute of layer
    l; "sync" waits for every layer before the first kernel (the reference's
    disk_sync).  Returns ``engine.cacheblend``'s result plus the loader stats.
    """
    if mode not in ("async", "sync"):
        raise ValueError("mode is async or sync")
    check = blend.check_layer
    layers = list(range(check, engine.cfg.n_layers))
    blocks = loader.start([disk.path(d) for d in request.documents], layers)
    table = engine.compose_table(slot, blocks, first_slot=len(request.prefix))
    if mode == "sync":
        for l in layers:
            loader.wait_layer(l)
        engine.compose_layers(slot, table, check, engine.cfg.n_layers)
        hook = None
    else:
        def hook(layer: int) -> None:
            if layer >= check:
                loader.wait_layer(layer)
                engine.compose_layers(slot, table, layer, layer + 1)

    out = engine.cacheblend(ids, slot, prefix_tokens=len(request.prefix), suffix_tokens=len(request.suffix),
                            blend=blend, before_layer=hook)
    return out, loader
