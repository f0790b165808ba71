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
  1. AG -> QKV GEMM: the TMA producer reads every rank's normed shard
     directly from its buffer (peer-mapped over CUDA IPC; plain TMA loads, no
     multicast), own shard first, after a bounded wait on that shard's ready
     flag; epilogue = RoPE + local K/V cache write.
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
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch
import torch.distributed as dist

from .. import ops
from ..config import ModelConfig
from ..models.engine import B200Engine, EngineWeights, KVSlot, LayerWeights
from ..models.weights import GATE_UP_BLOCK

FLAG_X, FLAG_X2, FLAG_RS_O, FLAG_RS_D = 0, 1, 2, 3
FLAG_AR_O, FLAG_AR_D, FLAG_TOKEN, FLAG_TOKEN_EPOCH = 4, 5, 6, 7
FLAG_STAGE_X, FLAG_STAGE_X2 = 8, 9  # local: a peer shard has landed in the staging buffer
N_FLAG_KINDS = 10
TIMEOUT_NS = int(20e9)


class TPGroup:
    """Peer-mapped buffers shared by the ranks of one TP group."""

    def __init__(self, group=None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._opened: list[int] = []
        self._keep: list[torch.Tensor] = []

    def shared(self, nbytes: int) -> tuple[torch.Tensor, list[int]]:
        """Allocate nbytes on every rank; return (local buffer, device address of each rank's buffer)."""
        ext = ops.ext()
        buf, handle = ext.shared_empty(int(nbytes), self.device.index)
        self._keep.append(buf)
        handles = [None] * self.size
        dist.all_gather_object(handles, handle, group=self.group)
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(buf.data_ptr())
            else:
                p = ext.shared_open(h)
                self._opened.append(p)
                ptrs.append(p)
        return buf, ptrs

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

    def __init__(self, cfg: ModelConfig, weights: EngineWeights, group: TPGroup, *, max_rows: int,
                 max_positions: int = 65536) -> None:
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
        self.flag_buf, self.flag_ptrs = group.shared(N_FLAG_KINDS * self.tp * 4)
        self.flags = self.flag_buf.view(torch.int32).view(N_FLAG_KINDS, self.tp)
        # decode all-reduce receive slots [tp, 8 rows, d] fp32 (O and down)
        self.ar_o_buf, self.ar_o_ptrs = group.shared(self.tp * 8 * d * 4)
        self.ar_d_buf, self.ar_d_ptrs = group.shared(self.tp * 8 * d * 4)
        self.ar_counters = torch.zeros(2, dtype=torch.int32, device=group.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=group.device)
        self.epoch = 0
        self.token_epoch = 0
        # local staging of the gathered activations: every remote shard crosses
        # NVLink once (copy engine), the GEMM re-reads tiles from local memory
        self.stage_x = torch.empty(self.tp * R, d, device=group.device, dtype=torch.bfloat16)
        self.stage_x2 = torch.empty(self.tp * R, d, device=group.device, dtype=torch.bfloat16)
        self.side = torch.cuda.Stream(device=group.device)

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
    def prefill(self, ids: torch.Tensor, slot: KVSlot) -> tuple[torch.Tensor, int, int]:
        """Prefill ids (all ranks pass the same int32 device ids).

        Returns (this rank's final-normed hidden shard [rows, d], rows, padded
        length).  The shard owning row T-1 holds the last prompt row.
        """
        ext, eng, cfg, lc = self.ext, self.engine, self.full_cfg, self.lcfg
        T = ids.numel()
        rows = int(math.ceil(T / (self.tp * 128)) * 128)
        if rows > self.max_rows:
            raise ValueError("prompt exceeds the TP buffers")
        Tp = rows * self.tp
        if Tp > slot.capacity:
            raise ValueError("slot capacity below the padded prompt")
        d = cfg.d_model
        ids_p = torch.zeros(Tp, dtype=torch.int32, device=ids.device)
        ids_p[:T] = ids
        own = slice(self.rank * rows, (self.rank + 1) * rows)
        h = eng.ws.get("tp_h", (rows, d), torch.bfloat16)
        ext.embedding(ids_p[own], eng.w.embed, h)
        x = self.x_buf.view(torch.bfloat16)[: rows * d].view(rows, d)
        x2 = self.x2_buf.view(torch.bfloat16)[: rows * d].view(rows, d)
        recv_o = self.recv_o_buf.view(torch.bfloat16)[: self.tp * rows * d].view(self.tp, rows, d)
        recv_d = self.recv_d_buf.view(torch.bfloat16)[: self.tp * rows * d].view(self.tp, rows, d)
        ext.rmsnorm(h, None, eng.w.layers[0].ln1, cfg.rms_eps, x)
        pos = eng._arange("pos", Tp)
        q = eng.ws.get("q", (Tp, lc.q_size), torch.bfloat16)
        attn = eng.ws.get("attn", (Tp, lc.q_size), torch.bfloat16)
        act = eng.ws.get("act", (Tp, lc.ffn), torch.bfloat16)
        bn = eng.bn
        for layer, lw in enumerate(eng.w.layers):
            self.epoch += 1
            e = self.epoch
            self._signal_all(FLAG_X, e)
            bases = self._pull_shards(FLAG_X, FLAG_STAGE_X, self.x_ptrs, self.stage_x, rows, e)
            ext.gemm_ag_qkv(bases, rows, self.rank, self.flags[FLAG_STAGE_X], e, d, lw.w_qkv, q, slot.k(layer),
                            slot.v(layer), pos, pos, eng.rope, lc.n_heads, lc.n_kv_heads, bn)
            ext.attention_prefill(q, None, pos, slot.k(layer), slot.v(layer), None, Tp, lc.n_heads, eng.scale, attn)
            ext.gemm_rs(attn, lw.w_o, self.recv_o_ptrs, rows, self.rank, bn)
            self._signal_all(FLAG_RS_O, e)
            ext.rs_reduce(recv_o, self.flags[FLAG_RS_O], e, TIMEOUT_NS, self.status, h, h, lw.ln2, x2, cfg.rms_eps)
            self._signal_all(FLAG_X2, e)
            bases = self._pull_shards(FLAG_X2, FLAG_STAGE_X2, self.x2_ptrs, self.stage_x2, rows, e)
            ext.gemm_ag_swiglu(bases, rows, self.rank, self.flags[FLAG_STAGE_X2], e, d, lw.w_gu, act, bn)
            ext.gemm_rs(act, lw.w_down, self.recv_d_ptrs, rows, self.rank, bn)
            self._signal_all(FLAG_RS_D, e)
            nxt = eng.w.layers[layer + 1].ln1 if layer + 1 < len(eng.w.layers) else eng.w.norm
            ext.rs_reduce(recv_d, self.flags[FLAG_RS_D], e, TIMEOUT_NS, self.status, h, h, nxt, x, cfg.rms_eps)
        return x, rows, Tp

    # ------------------------------------------------------------- decode
    def first_token(self, x_shard: torch.Tensor, rows: int, T: int, *, max_new: int) -> None:
        """The owner of prompt row T-1 runs the LM head and sends the token to every rank."""
        eng, ext = self.engine, self.ext
        owner = (T - 1) // rows
        self.token_epoch += 1
        b = eng._decode_buffers(max_new)
        if self.rank == owner:
            lr = (T - 1) - owner * rows
            b["counter"].zero_()
            ext.gemv_argmax(x_shard[lr:lr + 1], eng.w.lm_head, None, self.full_cfg.rms_eps, b["pv"], b["pi"],
                            b["counter"], b["tok"], None, None, None, None, None)
            for r in range(self.tp):
                ext.peer_signal(self._flag_addr(r, FLAG_TOKEN, owner), 0, None, b["tok"][0:1])
            ext.peer_signal_many([self._flag_addr(r, FLAG_TOKEN_EPOCH, owner) for r in range(self.tp)],
                                 self.token_epoch)
        ext.wait_flag(self.flags[FLAG_TOKEN_EPOCH], owner, self.token_epoch, TIMEOUT_NS, self.status)
        tok = self.flags[FLAG_TOKEN, owner:owner + 1]
        ext.embedding(tok, eng.w.embed, b["h"][:1])
        b["log"][0:1].copy_(tok)
        b["gen"].fill_(1)
        b["counter"].zero_()
        # keep the monotonic step counter pos[3]; reset position / slot / view
        b["pos"][:3].fill_(T)

    def _decode_step(self, slot: KVSlot, splits: int) -> None:
        eng, ext, cfg, lc = self.engine, self.ext, self.full_cfg, self.lcfg
        b = eng._decode_buffers()
        h, pos = b["h"][:1], b["pos"]
        step = pos[3:4]
        mul = 2 * lc.n_layers
        ar_o = self.ar_o_buf.view(torch.float32)[: self.tp * cfg.d_model].view(self.tp, 1, cfg.d_model)
        ar_d = self.ar_d_buf.view(torch.float32)[: self.tp * cfg.d_model].view(self.tp, 1, cfg.d_model)
        fo = [self._flag_addr(r, FLAG_AR_O, self.rank) for r in range(self.tp)]
        fd = [self._flag_addr(r, FLAG_AR_D, self.rank) for r in range(self.tp)]
        for layer, lw in enumerate(eng.w.layers):
            ext.gemv_qkv(h, lw.w_qkv, lw.ln1, cfg.rms_eps, b["q"][:1], slot.k(layer), slot.v(layer), pos[0:1],
                         eng.rope, lc.n_heads, lc.n_kv_heads, slot=pos[1:2])
            ext.attention_decode(b["q"][:1], slot.k(layer), slot.v(layer), pos[0:1], lc.n_heads, eng.scale, splits,
                                 b["attn"][:1], ws=b["attn_ws"], counters=b["attn_cnt"])
            ext.gemv_allreduce(b["attn"][:1], lw.w_o, None, cfg.rms_eps, self.ar_o_ptrs, fo, self.rank,
                               2 * layer + 1, step, mul, self.ar_counters[0:1])
            ext.rs_reduce(ar_o, self.flags[FLAG_AR_O], 2 * layer + 1, TIMEOUT_NS, self.status, h, h, None, None,
                          cfg.rms_eps, step, mul)
            ext.gemv_swiglu(h, lw.w_gu, lw.ln2, cfg.rms_eps, b["act"][:1])
            ext.gemv_allreduce(b["act"][:1], lw.w_down, None, cfg.rms_eps, self.ar_d_ptrs, fd, self.rank,
                               2 * layer + 2, step, mul, self.ar_counters[1:2])
            ext.rs_reduce(ar_d, self.flags[FLAG_AR_D], 2 * layer + 2, TIMEOUT_NS, self.status, h, h, None, None,
                          cfg.rms_eps, step, mul)
        ext.gemv_argmax(h, eng.w.lm_head, eng.w.norm, cfg.rms_eps, b["pv"], b["pi"], b["counter"], b["tok"],
                        b["log"], b["gen"], eng.w.embed, h, pos, 4)

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

    def check_status(self) -> None:
        st = int(self.status.item())
        if st:
            raise RuntimeError(f"a tensor-parallel wait timed out (status {st})")

    def close(self) -> None:
        self.group.close()
