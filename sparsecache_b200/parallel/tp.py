"""Tensor-parallel Llama with the collectives fused into the GEMMs (NVLink peer memory).

Layout (one process per GPU, TP group of size tp):
  * column-parallel: QKV (a rank owns n_heads/tp query heads and
    n_kv_heads/tp KV heads) and gate/up (ffn/tp in 128-row blocks);
  * row-parallel: o_proj and down_proj (the matching K slices);
  * sequence-parallel activations between blocks: rank r owns prompt rows
    [r * rows, (r + 1) * rows) of the residual stream (rows a multiple of 128;
    the prompt is padded to tp * rows, padded rows sit after every real
    position so causal attention never reads them).

Per layer and rank (all inside ONE stream, no host sync, no NCCL):
  1. AG -> QKV GEMM: a side stream pulls every peer's normed shard into
     local staging with one copy-engine transfer over NVLink each (after a
     bounded device wait on the owner's ready flag), so a remote tile crosses
     NVLink once although every column tile of the GEMM reads it; the GEMM's
     TMA producer (plain loads of local memory, no multicast) starts on its
     own shard in place and reads each staged shard after a bounded wait on
     that shard's local staged flag; epilogue = RoPE + local K/V cache write.
  2. attention of the local heads over all rows.
  3. o_proj GEMM -> RS: the epilogue stores every fp32 partial tile into the
     receive slot of the rank that owns the rows (NVLink stores), then a
     signal kernel releases that owner's flag for this sender.
  4. owner reduction: bounded wait for all senders, fixed-order sum +
     residual, fused RMSNorm -> the shard the gate/up all-gather reads.
  5. AG -> gate/up GEMM (SwiGLU epilogue), 6. down GEMM -> RS, 7. reduction
     fused with the next layer's input RMSNorm.
Epoch-numbered flags only ever increase, so one flag word per (kind, sender)
serves every layer; buffer reuse is safe because each rank reaches the next
write of a buffer only after consuming data every peer produced after its
last read of it.

CacheBlend (``cacheblend``): the layers before the check layer and the check
layer run over every prompt row as in prefill; the check layer's QKV
epilogue also writes each row's deviation from the composed cache for the
local kv heads, every rank pushes those partials to every peer (copy engine)
and all ranks run the same top-k over the sum, so the active set is
identical everywhere.  The residual rows are then all-gathered once and each
rank keeps its share of the active rows, which run the later layers with the
same fused AG/RS layer body (K/V written at their own slots, keys = the whole
composed prompt).

Decode, verify and drafting steps (single-row GEMVs with a fused all-reduce)
share one device step counter ``pos[3]``: the all-reduce number k of a step
uses epoch ``step * ar_stride + k``, each step advances the counter once,
and every step (and every captured graph) holds an even number of
all-reduces so that the two receive buffers strictly alternate.
"""
from __future__ import annotations

import math
import os
from dataclasses import replace

import torch
import torch.distributed as dist

from .. import ops
from ..config import ModelConfig
from ..models.engine import (BATCH_L2_PREFETCH, DECODE_L2_PREFETCH, B200Engine, EngineWeights, KVSlot,
                             LayerWeights)
from ..models.weights import GATE_UP_BLOCK

FLAG_X, FLAG_X2, FLAG_RS_O, FLAG_RS_D = 0, 1, 2, 3
FLAG_AR_O, FLAG_AR_D, FLAG_TOKEN, FLAG_TOKEN_EPOCH = 4, 5, 6, 7
FLAG_STAGE_X, FLAG_STAGE_X2 = 8, 9  # local: a peer shard has landed in the staging buffer
FLAG_DEV, FLAG_H, FLAG_STAGE_H = 10, 11, 12  # CacheBlend: deviation partials, residual all-gather
N_FLAG_KINDS = 13
TIMEOUT_NS = int(20e9)
# decode all-reduce: a separate reduce kernel, launched programmatically behind
# the sending GEMV, sums the ranks' partials over its whole grid.  With
# SC_TP_FUSED_REDUCE=1 the sending GEMV's last CTA does the reduction instead
# (one kernel boundary less, but one CTA sums tp x d values): 3.00 vs 2.82 ms
# TPOT for 8B and 4.66 vs 4.40 ms for 20 70B layers at TP2 (B200, measured).
FUSED_REDUCE = os.environ.get("SC_TP_FUSED_REDUCE", "0") == "1"
# Guard bands around every peer-mapped buffer: peers write into these buffers
# from their kernels (partial tiles, all-reduce rows, flags), so an index bug
# shows up as a changed guard band, checked by ``TPGroup.check_canaries``.
CANARY_BYTES = 4096  # keeps the buffer start 4 KiB-aligned (TMA needs 16 B)
CANARY_VALUE = 0xA5


class TPGroup:
    """Peer-mapped buffers shared by the ranks of one TP group."""

    def __init__(self, group=None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._opened: list[int] = []
        self._keep: list[torch.Tensor] = []
        self._guards: list[tuple[torch.Tensor, int]] = []

    def shared(self, nbytes: int) -> tuple[torch.Tensor, list[int]]:
        """Allocate nbytes on every rank; return (local buffer, device address of each rank's buffer).

        Each allocation carries ``CANARY_BYTES`` of guard band on both sides;
        the returned buffer and addresses point past the leading band.
        """
        ext = ops.ext()
        nbytes, pad = int(nbytes), CANARY_BYTES
        raw, handle = ext.shared_empty(nbytes + 2 * pad, self.device.index)
        raw[:pad].fill_(CANARY_VALUE)
        raw[pad + nbytes:].fill_(CANARY_VALUE)
        self._keep.append(raw)
        self._guards.append((raw, nbytes))
        buf = raw[pad:pad + nbytes]
        handles = [None] * self.size
        dist.all_gather_object(handles, handle, group=self.group)
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(buf.data_ptr())
            else:
                p = ext.shared_open(h)
                self._opened.append(p)
                ptrs.append(p + pad)
        return buf, ptrs

    def check_canaries(self) -> list[int]:
        """Indices (allocation order) of shared buffers whose guard bands were overwritten."""
        pad = CANARY_BYTES
        return [i for i, (raw, n) in enumerate(self._guards)
                if not (bool((raw[:pad] == CANARY_VALUE).all()) and bool((raw[pad + n:] == CANARY_VALUE).all()))]

    def close(self) -> None:
        ext = ops.ext()
        for p in self._opened:
            ext.shared_close(p)
        self._opened.clear()


def shard_weights(full: EngineWeights, cfg: ModelConfig, rank: int, tp: int) -> EngineWeights:
    """Column/row-parallel slices of full engine weights for ``rank``."""
    D = cfg.head_dim
    hq, hkv, f = cfg.n_heads // tp, cfg.n_kv_heads // tp, cfg.ffn // tp
    blk = GATE_UP_BLOCK
    layers = []
    for lw in full.layers:
        q = lw.w_qkv[: cfg.q_size]
        k = lw.w_qkv[cfg.q_size: cfg.q_size + cfg.kv_size]
        v = lw.w_qkv[cfg.q_size + cfg.kv_size:]
        qkv = torch.cat((q[rank * hq * D:(rank + 1) * hq * D], k[rank * hkv * D:(rank + 1) * hkv * D],
                         v[rank * hkv * D:(rank + 1) * hkv * D])).contiguous()
        gu = lw.w_gu.view(cfg.ffn // blk, 2 * blk, -1)[rank * f // blk:(rank + 1) * f // blk]
        layers.append(LayerWeights(
            ln1=lw.ln1, w_qkv=qkv, w_o=lw.w_o[:, rank * hq * D:(rank + 1) * hq * D].contiguous(), ln2=lw.ln2,
            w_gu=gu.reshape(2 * f, -1).contiguous(), w_down=lw.w_down[:, rank * f:(rank + 1) * f].contiguous()))
    return EngineWeights(embed=full.embed, layers=layers, norm=full.norm, lm_head=full.lm_head)


def local_config(cfg: ModelConfig, tp: int) -> ModelConfig:
    if cfg.n_heads % tp or cfg.n_kv_heads % tp or cfg.ffn % (tp * GATE_UP_BLOCK):
        raise ValueError("heads, kv heads and ffn/128 must divide by the TP size")
    return replace(cfg, n_heads=cfg.n_heads // tp, n_kv_heads=cfg.n_kv_heads // tp, ffn=cfg.ffn // tp)


class TPEngine:
    """Sequence/tensor-parallel prefill over a TP group with fused collectives."""

    MAX_BATCH = 32  # rows of a batched decode step (skinny tensor-core GEMM limit)

    def __init__(self, cfg: ModelConfig, weights: EngineWeights, group: TPGroup, *, max_rows: int,
                 max_positions: int = 65536, verify_backend: str = "skinny") -> None:
        self.full_cfg = cfg
        self.tp = group.size
        self.rank = group.rank
        self.group = group
        self.lcfg = local_config(cfg, self.tp)
        # the local engine runs the per-rank kernels (attention, norms, decode)
        self.engine = B200Engine(self.lcfg, weights, group.device, max_positions=max_positions)
        self.ext = self.engine.ext
        self.max_rows = int(math.ceil(max_rows / 128) * 128)
        d = cfg.d_model
        R = self.max_rows
        self.x_buf, self.x_ptrs = group.shared(R * d * 2)
        self.x2_buf, self.x2_ptrs = group.shared(R * d * 2)
        # bf16 partials of the row-parallel GEMMs, one slot per sender
        self.recv_o_buf, self.recv_o_ptrs = group.shared(self.tp * R * d * 2)
        self.recv_d_buf, self.recv_d_ptrs = group.shared(self.tp * R * d * 2)
        self.h_buf, self.h_ptrs = group.shared(R * d * 2)  # residual shard (all-gathered by CacheBlend)
        # deviation partials of every rank: [tp][tp * R rows][2 * local kv heads] fp32
        self.dev_stride = self.tp * R * 2 * self.lcfg.n_kv_heads
        self.dev_buf, self.dev_ptrs = group.shared(self.tp * self.dev_stride * 4)
        self.flag_buf, self.flag_ptrs = group.shared(N_FLAG_KINDS * self.tp * 4)
        self.flags = self.flag_buf.view(torch.int32).view(N_FLAG_KINDS, self.tp)
        # decode all-reduce receive slots [tp, MAX_BATCH rows, d] fp32 (O and down)
        self.ar_o_buf, self.ar_o_ptrs = group.shared(self.tp * self.MAX_BATCH * d * 4)
        self.ar_d_buf, self.ar_d_ptrs = group.shared(self.tp * self.MAX_BATCH * d * 4)
        self.ar_counters = torch.zeros(2, dtype=torch.int32, device=group.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=group.device)
        self.epoch = 0
        self.token_epoch = 0
        # local staging of the gathered activations: every remote shard crosses
        # NVLink once (copy engine), the GEMM re-reads tiles from local memory
        self.stage_x = torch.empty(self.tp * R, d, device=group.device, dtype=torch.bfloat16)
        self.stage_x2 = torch.empty(self.tp * R, d, device=group.device, dtype=torch.bfloat16)
        self.side = torch.cuda.Stream(device=group.device)
        # epochs per device step: >= the all-reduces of any step kind (decode /
        # verify: 2 per layer; a drafting graph: 3 per draft token)
        self.ar_stride = 2 * cfg.n_layers + 64
        L = cfg.n_layers
        self.seed_layers = tuple(sorted({min(2, L - 1), L // 2, max(0, L - 3)})) if L >= 3 else tuple(range(L))
        # verify rows (M <= 8) on the tensor-core skinny GEMM ("skinny") or the
        # CUDA-core multi-row GEMV ("gemv"); every verify call uses the same one,
        # so a row's result never depends on how many rows were verified with it
        if verify_backend not in ("skinny", "gemv"):
            raise ValueError("verify_backend is skinny or gemv")
        self.verify_backend = verify_backend
        if verify_backend == "skinny":
            lc, w0 = self.lcfg, weights.layers[0]
            shapes = [tuple(w0.w_qkv.shape), tuple(w0.w_o.shape), tuple(w0.w_gu.shape), tuple(w0.w_down.shape),
                      tuple(weights.lm_head.shape)]
            need = max(int(self.ext.skinny_splits(n, k)) * n * 32 for n, k in shapes)
            self.skinny_ws = torch.empty(need, device=group.device, dtype=torch.float32)

    @classmethod
    def from_full(cls, cfg: ModelConfig, full: EngineWeights, group: TPGroup, **kw) -> "TPEngine":
        return cls(cfg, shard_weights(full, cfg, group.rank, group.size), group, **kw)

    # ---------------------------------------------------------- helpers
    def _flag_addr(self, owner: int, kind: int, sender: int) -> int:
        return self.flag_ptrs[owner] + 4 * (kind * self.tp + sender)

    def _signal_all(self, kind: int, epoch: int) -> None:
        """Release flag (kind, me) on every rank (self included), one launch."""
        self.ext.peer_signal_many([self._flag_addr(r, kind, self.rank) for r in range(self.tp)], epoch)

    def new_slot(self, capacity: int) -> KVSlot:
        return self.engine.new_slot(capacity)

    def _pull_shards(self, kind: int, stage_kind: int, src_ptrs: list[int], stage: torch.Tensor, rows: int,
                     epoch: int) -> list[int]:
        """Copy every peer's shard into local staging on the side stream.

        Per remote shard (nearest rank first): a bounded device wait for the
        owner's ready flag, one copy-engine transfer over NVLink, then a local
        release of flags[stage_kind][r].  Returns the shard bases the GEMM
        reads (own shard in place, remote shards from staging).
        """
        d = self.full_cfg.d_model
        nbytes = rows * d * 2
        bases = []
        main = torch.cuda.current_stream()
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            for i in range(1, self.tp):
                r = (self.rank + i) % self.tp
                self.ext.wait_flag(self.flags[kind], r, epoch, TIMEOUT_NS, self.status)
                dst = stage[r * rows:(r + 1) * rows]
                self.ext.memcpy_async(dst.data_ptr(), src_ptrs[r], nbytes)
                self.ext.peer_signal(self._flag_addr(self.rank, stage_kind, r), epoch)
        for r in range(self.tp):
            bases.append(src_ptrs[r] if r == self.rank else stage[r * rows:].data_ptr())
        return bases

    # ------------------------------------------------------------ prefill
    def _views(self, rows: int):
        d, tp = self.full_cfg.d_model, self.tp
        bf = torch.bfloat16
        return (self.x_buf.view(bf)[: rows * d].view(rows, d), self.x2_buf.view(bf)[: rows * d].view(rows, d),
                self.recv_o_buf.view(bf)[: tp * rows * d].view(tp, rows, d),
                self.recv_d_buf.view(bf)[: tp * rows * d].view(tp, rows, d))

    def _layer(self, layer: int, rows: int, pos: torch.Tensor, slots: torch.Tensor, n_keys: int,
               h: torch.Tensor, nxt_norm: torch.Tensor, slot: KVSlot, *, dev_part: torch.Tensor | None = None,
               dev_mode: int = 0, push=None) -> int:
        """One fused TP layer over tp * rows rows (this rank's residual shard ``h`` [rows, d]).

        The normed input shard must already be in ``x_buf``; on return the
        next layer's normed input (``nxt_norm``) is there.  Rows write K/V at
        cache ``slots`` with RoPE ``pos`` and attend causally (by position) to
        keys [0, n_keys).  With ``push`` (a ``PushTarget`` of a peer slot with
        this rank's local geometry) the QKV epilogue also stores the local kv
        heads' rows into it and the layer's flag is released right after the
        GEMM.  Returns the epoch used.
        """
        ext, eng, cfg, lc = self.ext, self.engine, self.full_cfg, self.lcfg
        d, n = cfg.d_model, rows * self.tp
        x, x2, recv_o, recv_d = self._views(rows)
        q = eng.ws.get("q", (n, lc.q_size), torch.bfloat16)
        attn = eng.ws.get("attn", (n, lc.q_size), torch.bfloat16)
        act = eng.ws.get("act", (n, lc.ffn), torch.bfloat16)
        lw = eng.w.layers[layer]
        bn = eng.bn
        self.epoch += 1
        e = self.epoch
        self._signal_all(FLAG_X, e)
        bases = self._pull_shards(FLAG_X, FLAG_STAGE_X, self.x_ptrs, self.stage_x, rows, e)
        ext.gemm_ag_qkv(bases, rows, self.rank, self.flags[FLAG_STAGE_X], e, d, lw.w_qkv, q, slot.k(layer),
                        slot.v(layer), pos, slots, eng.rope, lc.n_heads, lc.n_kv_heads, bn, dev_part, dev_mode,
                        push.k(layer) if push is not None else 0, push.v(layer) if push is not None else 0)
        if push is not None:
            ext.peer_signal(push.flag(layer), push.epoch)
        ext.attention_prefill(q, None, pos, slot.k(layer), slot.v(layer), None, n_keys, lc.n_heads, eng.scale, attn)
        ext.gemm_rs(attn, lw.w_o, self.recv_o_ptrs, rows, self.rank, bn)
        self._signal_all(FLAG_RS_O, e)
        ext.rs_reduce(recv_o, self.flags[FLAG_RS_O], e, TIMEOUT_NS, self.status, h, h, lw.ln2, x2, cfg.rms_eps)
        self._signal_all(FLAG_X2, e)
        bases = self._pull_shards(FLAG_X2, FLAG_STAGE_X2, self.x2_ptrs, self.stage_x2, rows, e)
        ext.gemm_ag_swiglu(bases, rows, self.rank, self.flags[FLAG_STAGE_X2], e, d, lw.w_gu, act, bn)
        ext.gemm_rs(act, lw.w_down, self.recv_d_ptrs, rows, self.rank, bn)
        self._signal_all(FLAG_RS_D, e)
        ext.rs_reduce(recv_d, self.flags[FLAG_RS_D], e, TIMEOUT_NS, self.status, h, h, nxt_norm, x, cfg.rms_eps)
        return e

    def _next_norm(self, layer: int) -> torch.Tensor:
        w = self.engine.w
        return w.layers[layer + 1].ln1 if layer + 1 < len(w.layers) else w.norm

    def _embed_shard(self, ids: torch.Tensor, T: int, slot: KVSlot) -> tuple[torch.Tensor, int, int, torch.Tensor]:
        """Pad the prompt to tp * rows (rows a multiple of 128), embed this rank's rows, norm into x_buf."""
        eng, cfg = self.engine, self.full_cfg
        rows = int(math.ceil(T / (self.tp * 128)) * 128)
        if rows > self.max_rows:
            raise ValueError("prompt exceeds the TP buffers")
        Tp = rows * self.tp
        if Tp > slot.capacity:
            raise ValueError("slot capacity below the padded prompt")
        d = cfg.d_model
        ids_p = eng.ws.get("tp_ids", (Tp,), torch.int32)
        ids_p.zero_()
        ids_p[:T] = ids
        own = slice(self.rank * rows, (self.rank + 1) * rows)
        h = self.h_buf.view(torch.bfloat16)[: rows * d].view(rows, d)
        self.ext.embedding(ids_p[own], eng.w.embed, h)
        x = self._views(rows)[0]
        self.ext.rmsnorm(h, None, eng.w.layers[0].ln1, cfg.rms_eps, x)
        return h, rows, Tp, eng._arange("pos", Tp)

    def prefill(self, ids: torch.Tensor, slot: KVSlot, *, push=None) -> tuple[torch.Tensor, int, int]:
        """Prefill ids (all ranks pass the same int32 device ids).

        Returns (this rank's final-normed hidden shard [rows, d], rows, padded
        length).  The shard owning row T-1 holds the last prompt row.  With
        ``push`` every layer's local K/V rows (padded rows included, they sit
        past the prompt) are stored into the peer slot as they are written.
        """
        T = ids.numel()
        h, rows, Tp, pos = self._embed_shard(ids, T, slot)
        if push is not None and push.capacity != slot.capacity:
            raise ValueError("the pushed slot must have the local slot's capacity")
        for layer in range(self.full_cfg.n_layers):
            self._layer(layer, rows, pos, pos, Tp, h, self._next_norm(layer), slot, push=push)
        return self._views(rows)[0], rows, Tp

    def cacheblend(self, ids: torch.Tensor, slot: KVSlot, *, prefix_tokens: int, suffix_tokens: int,
                   blend) -> tuple[torch.Tensor, int, int, dict]:
        """Tensor-parallel CacheBlend over the composed cache already in ``slot`` (local kv heads).

        Same protocol as ``B200Engine.cacheblend`` (full recompute below the
        check layer, deviation top-k at the check layer, active rows only
        above it).  Returns (this rank's final-normed shard of the active rows
        [rows_a, d], rows_a, A, metadata); active row A-1 is the last prompt row.
        """
        from ..cacheblend import recompute_count

        if len(blend.schedule) > 1:
            raise NotImplementedError("gradual filtering (several check layers) runs on the single-GPU engine")
        ext, eng, cfg, lc = self.ext, self.engine, self.full_cfg, self.lcfg
        T = ids.numel()
        raw_len = T - suffix_tokens
        n_doc = raw_len - prefix_tokens
        check = blend.check_layer
        if not 0 <= check < cfg.n_layers:
            raise ValueError("check_layer lies outside the model")
        k_sel = recompute_count(n_doc, blend.recompute_ratio)
        A = (prefix_tokens if blend.keep_prefix else 0) + k_sel + suffix_tokens
        h, rows, Tp, pos = self._embed_shard(ids, T, slot)
        d = cfg.d_model
        for layer in range(check):
            self._layer(layer, rows, pos, pos, Tp, h, self._next_norm(layer), slot)
        # ---- check layer over every row, with the deviation partials of the local kv heads
        dev_part = eng.ws.get("tp_dev", (Tp, 2 * lc.n_kv_heads), torch.float32)
        e = self._layer(check, rows, pos, pos, Tp, h, self._next_norm(check), slot, dev_part=dev_part,
                        dev_mode=blend.dev_mode)
        # push the partials to every rank (copy engine over NVLink), then one flag per sender
        nbytes = Tp * 2 * lc.n_kv_heads * 4
        for r in range(self.tp):
            ext.memcpy_async(self.dev_ptrs[r] + self.rank * self.dev_stride * 4, dev_part.data_ptr(), nbytes)
        self._signal_all(FLAG_DEV, e)
        # all-gather the residual rows while the selection runs
        self._signal_all(FLAG_H, e)
        main = torch.cuda.current_stream()
        self._pull_shards(FLAG_H, FLAG_STAGE_H, self.h_ptrs, self.stage_x, rows, e)
        with torch.cuda.stream(self.side):
            ext.memcpy_async(self.stage_x[self.rank * rows:].data_ptr(), h.data_ptr(), rows * d * 2)
        for r in range(self.tp):
            ext.wait_flag(self.flags[FLAG_DEV], r, e, TIMEOUT_NS, self.status)
        dev_all = self.dev_buf.view(torch.float32)
        active = eng._i32("active", Tp)
        n_active = eng._i32("n_active", 1)
        scores = eng.ws.get("scores", (max(1, n_doc),), torch.float32)
        checksum = eng.ws.get("checksum", (1,), torch.int64)
        ext.cacheblend_select(dev_all, lc.n_kv_heads, blend.dev_mode, T, prefix_tokens, raw_len, k_sel,
                              blend.keep_prefix, active, n_active, scores, checksum, n_parts=self.tp,
                              part_stride=self.dev_stride)
        # ---- active rows: rows_a per rank; padding rows write K/V past the prompt
        rows_a = int(math.ceil(A / (self.tp * 128)) * 128)
        Ap = rows_a * self.tp
        if rows_a > self.max_rows or T + (Ap - A) > slot.capacity:
            raise ValueError("active rows exceed the TP buffers / slot capacity")
        act = active[:A]
        slots_a = eng._i32("tp_slots_a", Ap)
        slots_a[:A].copy_(act)
        if Ap > A:
            ext.arange_i32(slots_a[A:], T)
        src = eng._i32("tp_src_a", rows_a)
        own = slice(self.rank * rows_a, (self.rank + 1) * rows_a)
        src.copy_(torch.where(slots_a[own] < T, slots_a[own], torch.zeros_like(slots_a[own])))
        h_a = eng.ws.get("tp_ha", (rows_a, d), torch.bfloat16)
        main.wait_stream(self.side)
        ext.gather_rows(self.stage_x[:Tp], src, h_a)
        x_a = self._views(rows_a)[0]
        ext.rmsnorm(h_a, None, self._next_norm(check), cfg.rms_eps, x_a)
        for layer in range(check + 1, cfg.n_layers):
            self._layer(layer, rows_a, slots_a, slots_a, T, h_a, self._next_norm(layer), slot)
        meta = {"active": act, "n_active": n_active, "checksum": checksum, "k_selected": k_sel,
                "document_tokens": n_doc, "active_rows": A, "rows_per_rank": rows_a}
        return x_a, rows_a, A, meta

    # ------------------------------------------------------------- decode
    def first_token(self, x_shard: torch.Tensor, rows: int, T: int, *, max_new: int,
                    last_row: int | None = None) -> torch.Tensor:
        """The owner of the last prompt row runs the LM head and sends the token to every rank.

        ``last_row`` is that row's index in the sharded layout (default T-1;
        after CacheBlend it is the last active row, A-1); the next token is at
        position T.  Returns the token's device view (int32 [1], in this
        rank's flag block).
        """
        eng, ext = self.engine, self.ext
        last = T - 1 if last_row is None else int(last_row)
        owner = last // rows
        self.token_epoch += 1
        b = eng._decode_buffers(max_new)
        if self.rank == owner:
            lr = last - owner * rows
            b["counter"].zero_()
            ext.gemv_argmax(x_shard[lr:lr + 1], eng.w.lm_head, None, self.full_cfg.rms_eps, b["pv"], b["pi"],
                            b["counter"], b["tok"], None, None, None, None, None)
            for r in range(self.tp):
                ext.peer_signal(self._flag_addr(r, FLAG_TOKEN, owner), 0, None, b["tok"][0:1])
            ext.peer_signal_many([self._flag_addr(r, FLAG_TOKEN_EPOCH, owner) for r in range(self.tp)],
                                 self.token_epoch)
        ext.wait_flag(self.flags[FLAG_TOKEN_EPOCH], owner, self.token_epoch, TIMEOUT_NS, self.status)
        tok = self.flags[FLAG_TOKEN, owner:owner + 1]
        self.seed_decode(tok, T, max_new=max_new)
        return tok

    def seed_decode(self, tok: torch.Tensor, T: int, *, max_new: int) -> None:
        """Start greedy decode from a first token (device int32 [1], same on every rank) at position T.

        Used after ``first_token`` and by a decode group whose prompt K/V and
        seed token were pushed by a prefill group."""
        eng, ext = self.engine, self.ext
        b = eng._decode_buffers(max_new)
        ext.embedding(tok, eng.w.embed, b["h"][:1])
        b["log"][0:1].copy_(tok)
        b["gen"].fill_(1)
        b["counter"].zero_()
        # keep the monotonic step counter pos[3]; reset position / slot / view
        b["pos"][:3].fill_(T)

    def allreduce(self, x: torch.Tensor, w: torch.Tensor, k: int, residual: torch.Tensor,
                  norm_w: torch.Tensor | None = None, skinny: bool = False) -> None:
        """residual += sum over ranks of x @ w^T (row-parallel GEMV, M <= 8 rows), fused over peer memory.

        ``k`` numbers the all-reduce inside the current device step (epoch
        ``pos[3] * ar_stride + k``); odd k use the O receive buffer and flags,
        even k the down buffer, so consecutive all-reduces alternate.
        """
        eng, ext, cfg = self.engine, self.ext, self.full_cfg
        b = eng._decode_buffers()
        M, d = x.shape[0], residual.shape[1]
        step = b["pos"][3:4]
        odd = k % 2 == 1
        buf, ptrs = (self.ar_o_buf, self.ar_o_ptrs) if odd else (self.ar_d_buf, self.ar_d_ptrs)
        kind = FLAG_AR_O if odd else FLAG_AR_D
        flags = [self._flag_addr(r, kind, self.rank) for r in range(self.tp)]
        counter = self.ar_counters[0:1] if odd else self.ar_counters[1:2]
        recv = buf.view(torch.float32)[: self.tp * M * d].view(self.tp, M, d)
        if skinny:
            if norm_w is not None:
                raise ValueError("the skinny all-reduce takes normalised rows")
            ext.skinny_allreduce(x, w, ptrs, flags, self.rank, k, step, self.ar_stride, counter, self.skinny_ws)
        elif FUSED_REDUCE:
            # the GEMV's last CTA waits for every rank's partial and adds the sum to the residual:
            # no separate reduce kernel (one kernel boundary less per all-reduce)
            ext.gemv_allreduce(x, w, norm_w, cfg.rms_eps, ptrs, flags, self.rank, k, step, self.ar_stride, counter,
                               recv=recv, wait_flags=self.flags[kind], residual=residual, timeout_ns=TIMEOUT_NS,
                               status=self.status)
            return
        else:
            ext.gemv_allreduce(x, w, norm_w, cfg.rms_eps, ptrs, flags, self.rank, k, step, self.ar_stride, counter)
        ext.rs_reduce(recv, self.flags[kind], k, TIMEOUT_NS, self.status, residual, residual, None, None,
                      cfg.rms_eps, step, self.ar_stride)

    def _decode_step(self, slot: KVSlot, splits: int, M: int = 1, *, verify: bool = False) -> None:
        """One target step over the M rows in h (decode: M = 1 with token feedback; verify: M rows).

        A verify step writes the M rows' K/V at positions pos[0].., leaves the
        argmax after every row in tok[:M], copies the residual rows after the
        seed layers into ``feat`` and advances only the step counter.
        """
        eng, ext, cfg, lc = self.engine, self.ext, self.full_cfg, self.lcfg
        b = eng._decode_buffers()
        h, pos = b["h"][:M], b["pos"]
        feat = eng.ws.get("tp_feat", (len(self.seed_layers), eng.MAX_ROWS, cfg.d_model), torch.bfloat16)
        if verify and self.verify_backend == "skinny":
            self._verify_rows_skinny(slot, splits, M, feat)
            return
        for layer, lw in enumerate(eng.w.layers):
            ext.gemv_qkv(h, lw.w_qkv, lw.ln1, cfg.rms_eps, b["q"][:M], slot.k(layer), slot.v(layer), pos[0:1],
                         eng.rope, lc.n_heads, lc.n_kv_heads, slot=pos[1:2])
            ext.attention_decode(b["q"][:M], slot.k(layer), slot.v(layer), pos[0:1], lc.n_heads, eng.scale, splits,
                                 b["attn"][:M], ws=b["attn_ws"], counters=b["attn_cnt"],
                                 l2_prefetch=[lw.w_o, lw.w_gu], l2_prefetch_bytes=DECODE_L2_PREFETCH)
            self.allreduce(b["attn"][:M], lw.w_o, 2 * layer + 1, h)
            ext.gemv_swiglu(h, lw.w_gu, lw.ln2, cfg.rms_eps, b["act"][:M])
            self.allreduce(b["act"][:M], lw.w_down, 2 * layer + 2, h)
            if verify and layer in self.seed_layers:
                feat[self.seed_layers.index(layer), :M].copy_(h)
        if verify:
            ext.gemv_argmax(h, eng.w.lm_head, eng.w.norm, cfg.rms_eps, b["pv"], b["pi"], b["counter"], b["tok"],
                            None, None, None, None, None)
            ext.bump_counter(pos[3:4])
        else:
            ext.gemv_argmax(h, eng.w.lm_head, eng.w.norm, cfg.rms_eps, b["pv"], b["pi"], b["counter"], b["tok"],
                            b["log"], b["gen"], eng.w.embed, h, pos, 4)

    def _verify_rows_skinny(self, slot: KVSlot, splits: int, M: int, feat: torch.Tensor) -> None:
        """A verify step on the tensor-core skinny GEMM: norm, QKV (RoPE + cache), attention,
        o + all-reduce, norm, gate/up SwiGLU, down + all-reduce per layer; final norm, logits, argmax."""
        eng, ext, cfg, lc = self.engine, self.ext, self.full_cfg, self.lcfg
        b = eng._decode_buffers()
        h, pos = b["h"][:M], b["pos"]
        x = eng.ws.get("sk_x", (eng.MAX_ROWS, cfg.d_model), torch.bfloat16)[:M]
        ws = self.skinny_ws
        for layer, lw in enumerate(eng.w.layers):
            ext.rmsnorm(h, None, lw.ln1, cfg.rms_eps, x)
            ext.skinny_qkv(x, lw.w_qkv, b["q"][:M], slot.k(layer), slot.v(layer), pos[0:1], eng.rope, lc.n_heads,
                           lc.n_kv_heads, ws, slot=pos[1:2])
            ext.attention_decode(b["q"][:M], slot.k(layer), slot.v(layer), pos[0:1], lc.n_heads, eng.scale, splits,
                                 b["attn"][:M], ws=b["attn_ws"], counters=b["attn_cnt"])
            self.allreduce(b["attn"][:M], lw.w_o, 2 * layer + 1, h, skinny=True)
            ext.rmsnorm(h, None, lw.ln2, cfg.rms_eps, x)
            ext.skinny_gemm(x, lw.w_gu, 2, b["act"][:M], None, ws)
            self.allreduce(b["act"][:M], lw.w_down, 2 * layer + 2, h, skinny=True)
            if layer in self.seed_layers:
                feat[self.seed_layers.index(layer), :M].copy_(h)
        ext.rmsnorm(h, None, eng.w.norm, cfg.rms_eps, x)
        logits = eng.ws.get("sk_logits", (eng.MAX_ROWS, cfg.vocab), torch.bfloat16)[:M]
        ext.skinny_gemm(x, eng.w.lm_head, 0, logits, None, ws)
        ext.row_argmax(logits, b["tok"])
        ext.bump_counter(pos[3:4])

    def set_rows_state(self, position: int) -> None:
        """Host write of the next rows' position / slot / key count (the step counter pos[3] is kept)."""
        self.engine._decode_buffers()["pos"][:3].fill_(int(position))

    def verify(self, slot: KVSlot, tokens: torch.Tensor, position: int, *, use_graph: bool = True) -> torch.Tensor:
        """Forward M <= 8 tokens (device int32, same on every rank) at positions position.. as one step.

        Returns the device argmax after every row; the residual rows after
        the seed layers are left in the ``tp_feat`` workspace for a drafter.
        """
        eng, ext = self.engine, self.ext
        M = int(tokens.numel())
        if not 1 <= M <= eng.MAX_ROWS:
            raise ValueError("verify handles 1..8 rows")
        b = eng._decode_buffers()
        splits = eng._decode_splits(slot.capacity)
        b["ids"][:M].copy_(tokens, non_blocking=True)
        ext.embedding(b["ids"][:M], eng.w.embed, b["h"][:M])
        self.set_rows_state(position)
        if not use_graph:
            self._decode_step(slot, splits, M, verify=True)
            return b["tok"][:M]
        key = ("tpv", id(slot), splits, M, self.verify_backend)
        graph = eng._graphs.get(key)
        if graph is None:
            # a real warm step (its K/V rows are rewritten by the next verify at
            # the same positions), then capture; the step counter keeps increasing
            saved = b["h"][:M].clone()
            self._decode_step(slot, splits, M, verify=True)
            b["h"][:M].copy_(saved)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._decode_step(slot, splits, M, verify=True)
            eng._graphs[key] = graph
        graph.replay()
        per_layer = 12 if self.verify_backend == "skinny" else 7
        ext.launches += per_layer * len(eng.w.layers) + (5 if self.verify_backend == "skinny" else 2)
        return b["tok"][:M]

    def decode_breakdown(self, slot: KVSlot, reps: int = 3) -> dict[str, float]:
        """Per-op device time of one eager decode step (ms, summed over layers, mean of ``reps``).

        CUDA events bracket each op of the step (qkv, attention, o + all-reduce
        send, o reduce, gate/up, down + all-reduce send, down reduce, LM head);
        every rank runs the same steps.  Events between kernels add small gaps,
        so the total exceeds the graph-replayed TPOT a little.
        """
        eng, ext, cfg, lc = self.engine, self.ext, self.full_cfg, self.lcfg
        splits = eng._decode_splits(slot.capacity)
        names = ("qkv", "attention", "o_allreduce_send", "o_reduce", "gate_up", "down_allreduce_send", "down_reduce",
                 "lm_head")
        acc = {n: 0.0 for n in names}
        orig_step = self._decode_step

        for _ in range(reps):
            marks: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

            class _Timed:  # wraps the extension: every call between two events
                def __getattr__(_s, name):
                    fn = getattr(ext, name)
                    label = {"gemv_qkv": "qkv", "attention_decode": "attention", "gemv_swiglu": "gate_up",
                             "gemv_argmax": "lm_head"}.get(name)
                    if name == "gemv_allreduce":
                        label = "o_allreduce_send" if sum(m[0].startswith("o_a") for m in marks) <= \
                            sum(m[0].startswith("down_a") for m in marks) else "down_allreduce_send"
                    if name == "rs_reduce":
                        label = "o_reduce" if sum(m[0] == "o_reduce" for m in marks) <= \
                            sum(m[0] == "down_reduce" for m in marks) else "down_reduce"
                    if label is None:
                        return fn

                    def call(*a, **k):
                        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
                        e0.record()
                        out = fn(*a, **k)
                        e1.record()
                        marks.append((label, e0, e1))
                        return out

                    return call

            self.ext = _Timed()
            try:
                orig_step(slot, splits)
            finally:
                self.ext = ext
            torch.cuda.synchronize()
            for label, e0, e1 in marks:
                acc[label] += e0.elapsed_time(e1) / reps
        return acc

    def decode(self, slot: KVSlot, n_steps: int, *, use_graph: bool = True) -> None:
        """Greedy decode across the TP group; every rank runs the same steps."""
        eng = self.engine
        splits = eng._decode_splits(slot.capacity)
        if not use_graph:
            for _ in range(n_steps):
                self._decode_step(slot, splits)
            return
        key = ("tp", id(slot), splits)
        graph = eng._graphs.get(key)
        if graph is None:
            # capture needs warm launch attributes but must not advance the
            # group's state: warm up with one real step, then roll back only
            # the local scalars (flags and the step counter keep increasing)
            b = eng._decode_buffers()
            saved = {k: b[k].clone() for k in ("h", "gen", "log", "tok")}
            saved_pos = b["pos"][:3].clone()
            self._decode_step(slot, splits)
            for k, v in saved.items():
                b[k].copy_(v)
            b["pos"][:3].copy_(saved_pos)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._decode_step(slot, splits)
            eng._graphs[key] = graph
        for _ in range(n_steps):
            graph.replay()

    # ------------------------------------------------------ batched decode
    def batch_slots(self, n_seq: int, capacity: int) -> list[KVSlot]:
        """``n_seq`` slots back to back in one buffer (a batched step addresses them by stride)."""
        if not 1 <= n_seq <= self.MAX_BATCH:
            raise ValueError(f"1..{self.MAX_BATCH} sequences per batched step")
        lc = self.lcfg
        per = lc.n_layers * 2 * lc.n_kv_heads * capacity * lc.head_dim
        buf = torch.empty(n_seq * per, dtype=torch.bfloat16, device=self.group.device)
        return [KVSlot.from_buffer(lc, capacity, buf[i * per:(i + 1) * per]) for i in range(n_seq)]

    def _batch_buffers(self) -> dict:
        eng, cfg, lc, B = self.engine, self.full_cfg, self.lcfg, self.MAX_BATCH
        ws = eng.ws
        if "bt_gen" not in ws.bufs:
            ws.bufs["bt_gen"] = torch.zeros(1, device=eng.device, dtype=torch.int64)
        steps = eng.MAX_DECODE_TOKENS
        return {"h": ws.get("bt_h", (B, cfg.d_model), torch.bfloat16),
                "x": ws.get("bt_x", (B, cfg.d_model), torch.bfloat16),
                "q": ws.get("bt_q", (B, lc.q_size), torch.bfloat16),
                "attn": ws.get("bt_attn", (B, lc.q_size), torch.bfloat16),
                "act": ws.get("bt_act", (B, lc.ffn), torch.bfloat16),
                "logits": ws.get("bt_logits", (B, cfg.vocab), torch.bfloat16),
                "tok": ws.get("bt_tok", (B,), torch.int32),
                "pos": ws.get("bt_pos", (B,), torch.int32),
                "gen": ws.bufs["bt_gen"],
                "log": ws.get("bt_log", (steps, B), torch.int32)}

    def start_batch(self, slots: list[KVSlot], first_tokens, positions, *, max_new: int) -> None:
        """Seed a batched decode: sequence b has produced ``first_tokens[b]`` at ``positions[b]``."""
        B = len(slots)
        if self.verify_backend != "skinny":
            raise ValueError("batched decode runs on the skinny tensor-core GEMM")
        if len(first_tokens) != B or len(positions) != B:
            raise ValueError("one first token and one position per sequence")
        bb = self._batch_buffers()
        if max_new > bb["log"].shape[0]:
            raise ValueError("max_new exceeds the batched token log")
        bb["tok"][:B].copy_(torch.as_tensor(list(first_tokens), dtype=torch.int32))
        bb["pos"][:B].copy_(torch.as_tensor(list(positions), dtype=torch.int32))
        bb["log"][0, :B].copy_(bb["tok"][:B])
        bb["gen"].fill_(1)
        self.ext.embedding(bb["tok"][:B], self.engine.w.embed, bb["h"][:B])

    def _batch_step(self, slots: list[KVSlot], splits: int) -> None:
        """One greedy step for every sequence (row b = sequence b, its own position and slot)."""
        eng, ext, cfg, lc = self.engine, self.ext, self.full_cfg, self.lcfg
        B = len(slots)
        bb = self._batch_buffers()
        h, x, pos_rows = bb["h"][:B], bb["x"][:B], bb["pos"][:B]
        stride = (slots[1].data.data_ptr() - slots[0].data.data_ptr()) // 2 if B > 1 else 0
        ws = self.skinny_ws
        b = eng._decode_buffers()
        for layer, lw in enumerate(eng.w.layers):
            ext.rmsnorm(h, None, lw.ln1, cfg.rms_eps, x)
            ext.skinny_qkv(x, lw.w_qkv, bb["q"][:B], slots[0].k(layer), slots[0].v(layer), pos_rows, eng.rope,
                           lc.n_heads, lc.n_kv_heads, ws, pos_rows=pos_rows, seq_stride=stride)
            # every sequence in one launch: row b reads its own slot (stride apart) at pos_rows[b]
            ext.attention_decode(bb["q"][:B], slots[0].k(layer), slots[0].v(layer), pos_rows, lc.n_heads, eng.scale,
                                 splits, bb["attn"][:B], pos_rows=pos_rows, seq_stride=stride,
                                 l2_prefetch=[lw.w_o, lw.w_gu], l2_prefetch_bytes=BATCH_L2_PREFETCH)
            self.allreduce(bb["attn"][:B], lw.w_o, 2 * layer + 1, h, skinny=True)
            ext.rmsnorm(h, None, lw.ln2, cfg.rms_eps, x)
            ext.skinny_gemm(x, lw.w_gu, 2, bb["act"][:B], None, ws)
            self.allreduce(bb["act"][:B], lw.w_down, 2 * layer + 2, h, skinny=True)
        ext.rmsnorm(h, None, eng.w.norm, cfg.rms_eps, x)
        ext.skinny_gemm(x, eng.w.lm_head, 0, bb["logits"][:B], None, ws)
        ext.row_argmax(bb["logits"][:B], bb["tok"])
        bb["log"][:, :B].index_copy_(0, bb["gen"], bb["tok"][:B].view(1, B))
        bb["gen"].add_(1)
        pos_rows.add_(1)
        ext.embedding(bb["tok"][:B], eng.w.embed, h)
        ext.bump_counter(b["pos"][3:4])

    def decode_batch(self, slots: list[KVSlot], n_steps: int, *, use_graph: bool = True) -> None:
        """``n_steps`` batched greedy steps from the state ``start_batch`` (or earlier steps) left."""
        eng = self.engine
        if len({s.capacity for s in slots}) != 1:
            raise ValueError("batched slots share one capacity")
        splits = eng._batch_splits(slots[0].capacity, len(slots), self.lcfg.n_kv_heads)
        if not use_graph:
            for _ in range(n_steps):
                self._batch_step(slots, splits)
            return
        key = ("tpb", tuple(id(s) for s in slots), splits)
        graph = eng._graphs.get(key)
        if graph is None:
            bb = self._batch_buffers()
            saved = {k: bb[k].clone() for k in ("h", "tok", "pos", "gen", "log")}
            self._batch_step(slots, splits)  # warm step; the group's step counter keeps increasing
            for k, v in saved.items():
                bb[k].copy_(v)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._batch_step(slots, splits)
            eng._graphs[key] = graph
        for _ in range(n_steps):
            graph.replay()
        per_layer = 11
        self.ext.launches += n_steps * (per_layer * len(eng.w.layers) + 6)

    def batch_tokens(self, n_seq: int, n_tokens: int) -> list[list[int]]:
        """Host copy of the batched token log: tokens[b] = sequence b's first ``n_tokens`` tokens."""
        log = self._batch_buffers()["log"][:n_tokens, :n_seq].cpu()
        return [log[:, b].tolist() for b in range(n_seq)]

    def check_status(self) -> None:
        st = int(self.status.item())
        if st:
            raise RuntimeError(f"a tensor-parallel wait timed out (status {st})")

    def close(self) -> None:
        self.group.close()
