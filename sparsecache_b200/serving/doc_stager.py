"""Stage-by-stage H2D staging of reusable document KV from the pinned host tier.

Progressive reuse serves a request while its documents are still arriving:
documents are laid out in ranked order and stage ``s`` holds the ranked
prefix ``documents[:count_s]``.  ``PinnedDocumentStager`` copies each stage's
NEW documents from pinned host memory into a device arena on its own copy
stream, bracketed by CUDA events, and makes the compute stream wait on a
stage's end event before that stage's compose reads it.

Overlapped staging launches the copy of stage s+1 as soon as stage s is
waited on, so the transfer runs under stage s's repair, drafting and
verification; serial staging launches each stage's copy only when the stage
starts.  ``finish`` reports per-stage bytes and copy-engine times.

Behaviour of the reference's ReusableDocumentKVStager
(experiments/reuse_cacheblend_pipeline.py:62-191) and of its overlapped vs
serial runs (:896-930, :1181-1252).  Only the layers the consumer reads are
copied (CacheBlend recomputes the layers below its check layer, so their K/V
never crosses PCIe); a document's layers [layer_begin, L) are one contiguous
range of its block, so a document is one cudaMemcpyAsync.  The device blocks
keep the full [L, ...] shape so the composer addresses them like any other
block (the layers below layer_begin are never read).
"""
from __future__ import annotations

from typing import Any, Sequence

import torch


def ranked_prefix_stages(selected_sets: Sequence[set[int]]) -> list[tuple[int, ...]]:
    """New document indices of every stage; every stage must be a ranked prefix."""
    stages, seen = [], 0
    for selected in selected_sets:
        count = len(selected)
        if set(selected) != set(range(count)):
            raise ValueError("selected document stages must be ranked prefixes")
        if count < seen:
            raise ValueError("document stages must not shrink")
        stages.append(tuple(range(seen, count)))
        seen = count
    return stages


class PinnedDocumentStager:
    """Per-stage H2D copies of document K/V blocks ([L, 2, H_kv, n, D], pinned)."""

    def __init__(self, host_blocks: Sequence[torch.Tensor], selected_sets: Sequence[set[int]], *, device,
                 layer_begin: int = 0) -> None:
        if not host_blocks:
            raise ValueError("no documents to stage")
        for b in host_blocks:
            if b.device.type != "cpu" or not b.is_pinned():
                raise ValueError("staged document blocks must live in pinned host memory")
        self.device = torch.device(device)
        self.layer_begin = int(layer_begin)
        self.host = list(host_blocks)
        self.stages = ranked_prefix_stages(selected_sets)
        if self.stages and sum(map(len, self.stages)) != len(host_blocks):
            raise ValueError("the last stage must contain every document")
        self.stream = torch.cuda.Stream(device=self.device)
        sizes = [h.numel() for h in self.host]
        arena = torch.empty(sum(sizes), dtype=self.host[0].dtype, device=self.device)
        self.device_blocks, off = [], 0
        for h, n in zip(self.host, sizes):
            self.device_blocks.append(arena[off:off + n].view(h.shape))
            off += n
        self._arena = arena
        self.starts = [torch.cuda.Event(enable_timing=True) for _ in self.stages]
        self.ends = [torch.cuda.Event(enable_timing=True) for _ in self.stages]
        self.launched = [False] * len(self.stages)

    def stage_bytes(self, stage: int) -> int:
        lb = self.layer_begin
        return sum(self.host[i][lb:].numel() * self.host[i].element_size() for i in self.stages[stage])

    def launch(self, stage: int) -> None:
        """Queue the stage's new documents on the copy stream (idempotent).

        Earlier stages that were never launched are queued first: a stage's
        view is the whole ranked prefix, so its documents must all arrive.
        """
        if self.launched[stage]:
            return
        for earlier in range(stage):
            if not self.launched[earlier]:
                self.launch(earlier)
        # the arena may still be read by compute work queued before this
        # launch (an earlier request's stages): order the copies after it
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.starts[stage].record(self.stream)
            for i in self.stages[stage]:
                lb = self.layer_begin
                self.device_blocks[i][lb:].copy_(self.host[i][lb:], non_blocking=True)
            self.ends[stage].record(self.stream)
        self.launched[stage] = True

    def wait(self, stage: int) -> None:
        """Make the current (compute) stream wait for the stage's copies (and the earlier stages')."""
        if not self.launched[stage]:
            raise RuntimeError(f"stage {stage} was not launched")
        # one copy stream in launch order: the stage's end event follows every earlier copy
        torch.cuda.current_stream(self.device).wait_event(self.ends[stage])

    def arrive(self, stage: int, *, overlap: bool) -> None:
        """Stage ``stage`` is needed now: overlapped staging also starts the next one."""
        self.launch(stage)
        self.wait(stage)
        if overlap and stage + 1 < len(self.stages):
            self.launch(stage + 1)

    def blocks(self, stage: int) -> list[torch.Tensor]:
        """Device blocks of the stage's documents (the ranked prefix); layers from layer_begin are valid."""
        count = sum(len(s) for s in self.stages[: stage + 1])
        return self.device_blocks[:count]

    def finish(self) -> dict[str, Any]:
        self.stream.synchronize()
        done = [s for s, on in enumerate(self.launched) if on]
        h2d = [self.starts[s].elapsed_time(self.ends[s]) for s in done]
        nbytes = [self.stage_bytes(s) for s in done]
        return {"launched_stages": len(done), "stage_bytes": nbytes, "stage_h2d_ms": h2d,
                "total_bytes": sum(nbytes), "total_h2d_ms": sum(h2d),
                "first_stage_h2d_ms": h2d[0] if h2d else None,
                "h2d_gbps": (sum(nbytes) / (sum(h2d) * 1e6)) if h2d and sum(h2d) > 0 else None}
