"""B200 inference engine: a Llama decoder driven entirely by the sm_100a kernels.

Data layout (chosen for the kernels, not translated from the reference):
  * weights: one fused QKV matrix, gate/up interleaved in 128-row blocks,
    bf16, contiguous, resident in HBM (weights.py);
  * KV cache: one contiguous [L, 2, H_kv, capacity, 128] bf16 buffer per
    serving slot.  Slots are positions, so a composed document cache, the
    CacheBlend scatter and the decode append all address the same buffer
    and the decode CUDA graph can be captured once per slot;
  * RoPE: one fp32 (cos, sin) table indexed by position, shared by the QKV
    epilogue, the decode GEMV and the composer.

Passes:
  * ``prefill``         full causal prefill (also the document producer and
                        the direct-reuse suffix prefill);
  * ``cacheblend``      the CacheBlend selective recompute (layers < check:
                        all rows; check layer: fused deviation epilogue +
                        radix top-k select; later layers: active rows only,
                        fresh K/V scattered in the QKV epilogue);
  * ``decode``          greedy decode, one CUDA graph per step: 5 launches
                        per layer plus the fused LM-head/argmax/embedding
                        feedback kernel.  The position, the token and the
                        token log live on the device; the host reads the
                        tokens once at the end.
Reference behaviour: modeling.py:33-417, reuse_cacheblend_pipeline.py:322-893.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from .. import ops
from ..config import CacheBlendConfig, ModelConfig
from ..rope import rope_table
from .weights import fuse_qkv, interleave_gate_up


@dataclass
class LayerWeights:
    ln1: torch.Tensor
    w_qkv: torch.Tensor
    w_o: torch.Tensor
    ln2: torch.Tensor
    w_gu: torch.Tensor
    w_down: torch.Tensor


@dataclass
class EngineWeights:
    embed: torch.Tensor
    layers: list[LayerWeights]
    norm: torch.Tensor
    lm_head: torch.Tensor

    @staticmethod
    def random(config: ModelConfig, *, seed: int, device, std: float = 0.02) -> "EngineWeights":
        """Seeded random bf16 weights generated directly on the device."""
        gen = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16

        def mat(rows, cols):
            w = torch.empty(rows, cols, device=device, dtype=bf)
            w.normal_(0.0, std, generator=gen)
            return w

        def ones(n):
            return torch.ones(n, device=device, dtype=bf)

        d, f = config.d_model, config.ffn
        layers = [
            LayerWeights(
                ln1=ones(d),
                w_qkv=mat(config.qkv_rows, d),
                w_o=mat(d, config.q_size),
                ln2=ones(d),
                w_gu=mat(2 * f, d),
                w_down=mat(d, f),
            )
            for _ in range(config.n_layers)
        ]
        return EngineWeights(embed=mat(config.vocab, d), layers=layers, norm=ones(d), lm_head=mat(config.vocab, d))

    @staticmethod
    def from_oracle(model, device) -> "EngineWeights":
        """Convert a LlamaOracle's parameters into the kernel layout (bf16)."""
        bf = torch.bfloat16

        def t(x):
            return x.detach().to(device=device, dtype=bf).contiguous()

        layers = []
        for layer in model.layers:
            layers.append(
                LayerWeights(
                    ln1=t(layer.input_layernorm.weight),
                    w_qkv=t(fuse_qkv(layer.q_proj.weight, layer.k_proj.weight, layer.v_proj.weight)),
                    w_o=t(layer.o_proj.weight),
                    ln2=t(layer.post_attention_layernorm.weight),
                    w_gu=t(interleave_gate_up(layer.gate_proj.weight, layer.up_proj.weight)),
                    w_down=t(layer.down_proj.weight),
                )
            )
        return EngineWeights(
            embed=t(model.embed_tokens.weight), layers=layers, norm=t(model.norm.weight), lm_head=t(model.lm_head.weight)
        )


class KVSlot:
    """A serving slot: one contiguous KV buffer of fixed capacity."""

    def __init__(self, config: ModelConfig, capacity: int, device) -> None:
        self.capacity = int(capacity)
        self.data = torch.empty(
            config.n_layers, 2, config.n_kv_heads, self.capacity, config.head_dim, device=device, dtype=torch.bfloat16
        )

    def k(self, layer: int) -> torch.Tensor:
        return self.data[layer, 0]

    def v(self, layer: int) -> torch.Tensor:
        return self.data[layer, 1]

    def nbytes(self) -> int:
        return self.data.numel() * 2

    @classmethod
    def from_buffer(cls, config: ModelConfig, capacity: int, buffer: torch.Tensor) -> "KVSlot":
        """Wrap an existing device buffer (e.g. an IPC-exported one) as a slot."""
        slot = cls.__new__(cls)
        slot.capacity = int(capacity)
        shape = (config.n_layers, 2, config.n_kv_heads, slot.capacity, config.head_dim)
        n = math.prod(shape)
        slot.data = buffer.view(torch.bfloat16)[:n].view(*shape)
        return slot

    @staticmethod
    def nbytes_for(config: ModelConfig, capacity: int) -> int:
        return config.n_layers * 2 * config.n_kv_heads * int(capacity) * config.head_dim * 2


@dataclass
class PushTarget:
    """A peer GPU's slot (mapped into this process) that prefill pushes K/V into.

    ``base`` / ``flags`` are device addresses valid in this process (CUDA IPC
    mappings of the decode GPU's buffers); after layer l's K/V rows are
    stored, ``flags[l]`` is released with ``epoch``.
    """

    base: int
    capacity: int
    flags: int
    epoch: int
    n_layers: int
    layer_elems: int  # n_kv_heads * capacity * head_dim

    def k(self, layer: int) -> int:
        return self.base + (layer * 2 + 0) * self.layer_elems * 2

    def v(self, layer: int) -> int:
        return self.base + (layer * 2 + 1) * self.layer_elems * 2

    def flag(self, index: int) -> int:
        return self.flags + 4 * index


# decode attention cross-cluster merge scratch per kv head: [16 clusters][64 query
# vectors][max, sum, o[128]] fp32, and one ticket counter per 4-vector z-block
ATTN_WS_PER_KVH = 16 * 64 * 130
ATTN_CNT_PER_KVH = 16
# Bytes of the following projections' weights (o, then the start of gate/up)
# that decode attention may prefetch into L2 while its key loop runs (the loop
# reads a few MB of K/V and leaves HBM mostly idle).  Off by default: with
# 64 MB the 8B greedy step measured slower (3.28 vs 3.19 ms per token).
DECODE_L2_PREFETCH = int(os.environ.get("SC_DECODE_L2_PREFETCH", "0"))
BATCH_L2_PREFETCH = int(os.environ.get("SC_BATCH_L2_PREFETCH", "0"))
# Row counts run on the token-column GEMM (weights as the MMA's M, tokens as
# its N): CacheBlend's active rows.  SC_WIDE_GEMM=0 keeps them on row tiles.
WIDE_ROWS = (65, 512)
USE_WIDE_GEMM = os.environ.get("SC_WIDE_GEMM", "1") != "0"


class _Workspace:
    """Grow-only device scratch buffers, reused across calls (no per-call allocation)."""

    def __init__(self, device) -> None:
        self.device = device
        self.bufs: dict[str, torch.Tensor] = {}

    def get(self, name: str, shape, dtype) -> torch.Tensor:
        numel = math.prod(shape)
        buf = self.bufs.get(name)
        if buf is None or buf.numel() < numel or buf.dtype != dtype:
            buf = torch.empty(max(numel, 1), device=self.device, dtype=dtype)
            self.bufs[name] = buf
        return buf[:numel].view(*shape)


class _CountingExt:
    """Proxy over the extension that counts kernel launches issued from the host."""

    _NOT_KERNELS = {"status", "num_sms", "gemv_argmax_grid", "attention_decode_cluster", "attention_decode_outer",
                    "skinny_splits", "attention_prefill_splits", "wide_plan", "set_wide_stream_k", "set_attention_prefill_splits",
                    "shared_empty",
                    "shared_open", "shared_close"}
    _MULTI = {"gemm_store", "gemm_residual", "skinny_gemm", "skinny_qkv", "skinny_allreduce", "attention_prefill",
              "wide_swiglu", "wide_residual", "wide_qkv"}

    def __init__(self, ext) -> None:
        self._ext = ext
        self.launches = 0

    def __getattr__(self, name):
        fn = getattr(self._ext, name)
        if name in self._NOT_KERNELS or not callable(fn):
            return fn

        def counted(*args, **kwargs):
            out = fn(*args, **kwargs)
            # ops that may issue several kernels return how many they launched
            self.launches += out if isinstance(out, int) and name in self._MULTI else 1
            return out

        return counted


class B200Engine:
    """Kernel-driven Llama forward passes on one GPU."""

    def __init__(self, config: ModelConfig, weights: EngineWeights, device, *, max_positions: int | None = None) -> None:
        ops.require_on_gpu()
        self.cfg = config
        self.w = weights
        self.device = torch.device(device)
        self.ext = _CountingExt(ops.ext())
        self.max_positions = int(max_positions or min(config.max_positions, 65536))
        self.rope = rope_table(config, self.max_positions, self.device)
        self.ws = _Workspace(self.device)
        self.scale = 1.0 / math.sqrt(config.head_dim)
        self.num_sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self._graphs: dict[tuple, torch.cuda.CUDAGraph] = {}
        self.bn = 256

    # ----------------------------------------------------------- helpers
    @classmethod
    def random(cls, config: ModelConfig, *, seed: int = 0, device="cuda", **kw) -> "B200Engine":
        return cls(config, EngineWeights.random(config, seed=seed, device=device), device, **kw)

    @classmethod
    def from_oracle(cls, model, device="cuda", **kw) -> "B200Engine":
        return cls(model.config, EngineWeights.from_oracle(model, device), device, **kw)

    def new_slot(self, capacity: int) -> KVSlot:
        return KVSlot(self.cfg, capacity, self.device)

    def _i32(self, name: str, n: int) -> torch.Tensor:
        return self.ws.get(name, (n,), torch.int32)

    def _arange(self, name: str, n: int, start: int = 0) -> torch.Tensor:
        t = self._i32(name, n)
        self.ext.arange_i32(t, start)
        return t

    # -------------------------------------------------------- layer body
    def _attn_mlp(
        self,
        layer: int,
        h: torch.Tensor,
        q: torch.Tensor,
        slot: KVSlot,
        *,
        q_rows: torch.Tensor | None,
        qpos: torch.Tensor,
        n_keys: int,
        kpos: torch.Tensor | None,
        n_rows: int,
        next_norm: torch.Tensor | None = None,
    ) -> None:
        """attention over the slot's keys, o_proj + residual, then the MLP block (in place on h).

        The post-attention RMSNorm is produced by the o_proj call (fused into
        its split-K reduce when it splits); with ``next_norm`` the down_proj
        call also leaves RMSNorm(h) with that weight in the ``x`` workspace,
        for the next layer's QKV (``_full_layer(..., x_ready=True)``)."""
        cfg, lw, ext = self.cfg, self.w.layers[layer], self.ext
        attn = self.ws.get("attn", (n_rows, cfg.q_size), torch.bfloat16)
        # few query rows (CacheBlend's active set) leave SMs idle: the kernel
        # splits the keys over several CTAs and merges fp32 partials from here
        split_ws = (self.ws.get("attn_split", (4 * self.ATTN_SPLIT_ROWS * cfg.n_heads * 132,), torch.float32)
                    if n_rows <= self.ATTN_SPLIT_ROWS else None)
        ext.attention_prefill(q, q_rows, qpos, slot.k(layer), slot.v(layer), kpos, n_keys, cfg.n_heads, self.scale, attn,
                              ws=split_ws)
        x = self.ws.get("x", (n_rows, cfg.d_model), torch.bfloat16)
        act = self.ws.get("act", (n_rows, cfg.ffn), torch.bfloat16)
        if self._wide(n_rows):
            ext.wide_residual(attn, lw.w_o, h, h, norm_w=lw.ln2, eps=cfg.rms_eps, norm_out=x)
            ext.wide_swiglu(x, lw.w_gu, act)
            if next_norm is None:
                ext.wide_residual(act, lw.w_down, h, h)
            else:
                ext.wide_residual(act, lw.w_down, h, h, norm_w=next_norm, eps=cfg.rms_eps, norm_out=x)
            return
        ext.gemm_residual(attn, lw.w_o, h, h, self.bn, norm_w=lw.ln2, eps=cfg.rms_eps, norm_out=x)
        ext.gemm_swiglu(x, lw.w_gu, act, self.bn)
        if next_norm is None:
            ext.gemm_residual(act, lw.w_down, h, h, self.bn)
        else:
            ext.gemm_residual(act, lw.w_down, h, h, self.bn, norm_w=next_norm, eps=cfg.rms_eps, norm_out=x)

    def _wide(self, rows: int) -> bool:
        """Whether ``rows`` token rows run on the token-column GEMM (every projection of the
        layer must tile: 128-row weight tiles, 256-row gate/up blocks, 64-deep k-blocks)."""
        cfg = self.cfg
        return (USE_WIDE_GEMM and WIDE_ROWS[0] <= rows <= WIDE_ROWS[1] and cfg.d_model % 128 == 0
                and cfg.ffn % 128 == 0 and cfg.d_model % 64 == 0 and cfg.q_size % 64 == 0 and cfg.d_model <= 8192)

    def _qkv_bn(self, rows: int) -> int:
        """128-column tiles when 256-column tiles would leave SMs idle (small M)."""
        tiles = -(-rows // 128) * -(-self.cfg.qkv_rows // 256)
        return 128 if tiles < self.num_sms else self.bn

    def _next_ln1(self, layer: int) -> torch.Tensor | None:
        """Input-norm weight of the layer after ``layer`` (None after the last layer)."""
        return self.w.layers[layer + 1].ln1 if layer + 1 < len(self.w.layers) else None

    def _full_layer(self, layer: int, h: torch.Tensor, slot: KVSlot, pos: torch.Tensor, slots: torch.Tensor,
                    n_keys: int, kpos: torch.Tensor | None, dev_part=None, dev_mode: int = 0,
                    push: PushTarget | None = None, x_ready: bool = False) -> torch.Tensor:
        """Norm + fused QKV/RoPE/scatter for every row of h; returns q.

        With ``push`` the QKV epilogue also stores every K/V row into the
        peer GPU's slot, and the layer's ready flag is released right after,
        while this GPU goes on with the layer's attention and MLP.
        """
        cfg, lw, ext = self.cfg, self.w.layers[layer], self.ext
        n = h.shape[0]
        x = self.ws.get("x", (n, cfg.d_model), torch.bfloat16)
        if not x_ready:  # else the previous layer's down_proj left RMSNorm(h) in x
            ext.rmsnorm(h, None, lw.ln1, cfg.rms_eps, x)
        q = self.ws.get("q", (n, cfg.q_size), torch.bfloat16)
        if dev_part is None and push is None and self._wide(n):
            ext.wide_qkv(x, lw.w_qkv, q, slot.k(layer), slot.v(layer), pos, slots, self.rope, cfg.n_heads,
                         cfg.n_kv_heads)
            return q
        ext.gemm_qkv(x, lw.w_qkv, q, slot.k(layer), slot.v(layer), pos, slots, self.rope,
                     cfg.n_heads, cfg.n_kv_heads, dev_part, dev_mode, self._qkv_bn(n),
                     push.k(layer) if push else 0, push.v(layer) if push else 0)
        if push is not None:
            ext.peer_signal(push.flag(layer), push.epoch)
        return q

    # ----------------------------------------------------------- compose
    def compose(self, slot: KVSlot, blocks, *, first_slot: int, layer_begin: int = 0,
                source_positions=None, target_positions=None, layer_end: int | None = None) -> None:
        """Gather document K/V blocks into ``slot`` after ``first_slot`` and re-rotate keys.

        ``blocks`` are [L, 2, H_kv, n, D] tensors in HBM or pinned host memory
        (the kernel reads mapped host memory directly).  Document i lands at
        slots cursor..cursor+n-1; its keys move from source position
        ``source_positions[i]`` (0 for independently produced documents) to
        ``target_positions[i]`` (default: its slot).  Layers outside
        [layer_begin, layer_end) are skipped: CacheBlend recomputes the layers
        below the check layer fully.
        """
        table = self.compose_table(slot, blocks, first_slot=first_slot, source_positions=source_positions,
                                   target_positions=target_positions)
        self.compose_layers(slot, table, layer_begin, self.cfg.n_layers if layer_end is None else layer_end)

    def compose_table(self, slot: KVSlot, blocks, *, first_slot: int, source_positions=None,
                      target_positions=None) -> tuple[torch.Tensor, torch.Tensor, int]:
        """Device table of the composer: (docs [n, 6] int32, token offsets [n + 1], total tokens)."""
        rows, offsets, cursor = [], [0], first_slot
        for i, block in enumerate(blocks):
            n = int(block.shape[3])
            ptr = int(block.data_ptr())
            src = 0 if source_positions is None else int(source_positions[i])
            dst = cursor if target_positions is None else int(target_positions[i])
            rows.append([ptr & 0xFFFFFFFF, ptr >> 32, n, src, cursor, dst])
            offsets.append(offsets[-1] + n)
            cursor += n
        if cursor > slot.capacity:
            raise ValueError("composed documents exceed the slot capacity")
        table = torch.tensor(rows, dtype=torch.int64)
        table = torch.where(table >= 2**31, table - 2**32, table).to(torch.int32)
        host = torch.empty((len(rows) * 6 + len(offsets),), dtype=torch.int32, pin_memory=True)
        host[: len(rows) * 6] = table.reshape(-1)
        host[len(rows) * 6 :] = torch.tensor(offsets, dtype=torch.int32)
        dev = self.ws.get("compose_meta", (host.numel(),), torch.int32)
        dev.copy_(host, non_blocking=True)
        return dev[: len(rows) * 6].view(len(rows), 6), dev[len(rows) * 6 :], offsets[-1]

    def compose_layers(self, slot: KVSlot, table, layer_begin: int, layer_end: int) -> None:
        """Run the composer over layers [layer_begin, layer_end) of a ``compose_table``."""
        docs, offs, total = table
        self.ext.compose_relocate(docs, offs, total, layer_begin, layer_end, self.cfg.n_layers, slot.data,
                                  self.cfg.n_kv_heads, self.rope)

    # ------------------------------------------------------------ passes
    def embed(self, ids: torch.Tensor, name: str = "h") -> torch.Tensor:
        h = self.ws.get(name, (ids.numel(), self.cfg.d_model), torch.bfloat16)
        self.ext.embedding(ids, self.w.embed, h)
        return h

    def prefill(self, ids: torch.Tensor, slot: KVSlot, *, start: int = 0, kpos: torch.Tensor | None = None,
                push: PushTarget | None = None, layer_hook=None) -> torch.Tensor:
        """Causal prefill of ``ids`` (int32, device) at positions/slots start.. ; returns final hidden [T, d].

        Keys [0, start) already in the slot are visible (direct prefix reuse).
        ``push`` streams every layer's K/V to a decode GPU as it is written.
        ``layer_hook(layer, h)`` sees the input hidden rows of every layer
        (the residual stream, before that layer's norm) for feature capture.
        """
        T = ids.numel()
        if start + T > slot.capacity or start + T > self.max_positions:
            raise ValueError("prompt exceeds slot capacity / RoPE table")
        if push is not None and push.capacity != slot.capacity:
            raise ValueError("the pushed slot must have the local slot's capacity")
        h = self.embed(ids)
        pos = self._arange("pos", T, start)
        for layer in range(self.cfg.n_layers):
            if layer_hook is not None:
                layer_hook(layer, h)
            q = self._full_layer(layer, h, slot, pos, pos, start + T, kpos, push=push, x_ready=layer > 0)
            self._attn_mlp(layer, h, q, slot, q_rows=None, qpos=pos, n_keys=start + T, kpos=kpos, n_rows=T,
                           next_norm=self._next_ln1(layer))
        return h

    def cacheblend(
        self,
        ids: torch.Tensor,
        slot: KVSlot,
        *,
        prefix_tokens: int,
        suffix_tokens: int,
        blend: CacheBlendConfig,
        global_positions: torch.Tensor | None = None,
        before_layer=None,
    ) -> tuple[torch.Tensor, int, dict]:
        """Selective recompute over the composed cache already in ``slot``.

        Returns (hidden of the active rows [A, d], A, device-side metadata).
        The number of active rows A is known on the host (no sync):
        prefix (strict protocol) + ceil(ratio * N_doc) + suffix.
        ``before_layer(layer)`` runs before each layer's kernels are issued
        (layer-wise cache arrival: wait for the layer, compose it).
        """
        if len(blend.schedule) > 1:
            if before_layer is not None:
                raise ValueError("layer hooks are not supported with gradual filtering")
            return self._cacheblend_gradual(ids, slot, prefix_tokens=prefix_tokens, suffix_tokens=suffix_tokens,
                                            blend=blend, global_positions=global_positions)
        cfg, ext = self.cfg, self.ext
        T = ids.numel()
        raw_len = T - suffix_tokens
        n_doc = raw_len - prefix_tokens
        if T > slot.capacity:
            raise ValueError("prompt exceeds slot capacity")
        check = blend.check_layer
        if not 0 <= check < cfg.n_layers:
            raise ValueError("check_layer lies outside the model")
        from ..cacheblend import recompute_count

        k_sel = recompute_count(n_doc, blend.recompute_ratio)
        A = (prefix_tokens if blend.keep_prefix else 0) + k_sel + suffix_tokens
        h = self.embed(ids)
        rows = self._arange("rows", T)
        gpos = rows if global_positions is None else global_positions
        kpos = global_positions  # None -> key position == slot
        for layer in range(check):
            if before_layer is not None:
                before_layer(layer)
            q = self._full_layer(layer, h, slot, gpos, rows, T, kpos, x_ready=layer > 0)
            self._attn_mlp(layer, h, q, slot, q_rows=None, qpos=gpos, n_keys=T, kpos=kpos, n_rows=T,
                           next_norm=self._next_ln1(layer))
        # ---- check layer ----
        if before_layer is not None:
            before_layer(check)
        dev_part = self.ws.get("dev", (T, 2 * cfg.n_kv_heads), torch.float32)
        q = self._full_layer(check, h, slot, gpos, rows, T, kpos, dev_part, blend.dev_mode, x_ready=check > 0)
        active = self._i32("active", T)
        n_active = self._i32("n_active", 1)
        scores = self.ws.get("scores", (max(1, n_doc),), torch.float32)
        checksum = self.ws.get("checksum", (1,), torch.int64)
        ext.cacheblend_select(dev_part, cfg.n_kv_heads, blend.dev_mode, T, prefix_tokens, raw_len, k_sel,
                              blend.keep_prefix, active, n_active, scores, checksum)
        act_rows = active[:A]
        qpos_a = self._i32("qpos_a", A)
        ext.index_i32(gpos, act_rows, qpos_a)
        h_a = self.ws.get("h_a", (A, cfg.d_model), torch.bfloat16)
        ext.gather_rows(h, act_rows, h_a)
        self._attn_mlp(check, h_a, q, slot, q_rows=act_rows, qpos=qpos_a, n_keys=T, kpos=kpos, n_rows=A,
                       next_norm=self._next_ln1(check))
        # ---- later layers: active rows only ----
        for layer in range(check + 1, cfg.n_layers):
            if before_layer is not None:
                before_layer(layer)
            qa = self._full_layer(layer, h_a, slot, qpos_a, act_rows, T, kpos, x_ready=True)
            self._attn_mlp(layer, h_a, qa, slot, q_rows=None, qpos=qpos_a, n_keys=T, kpos=kpos, n_rows=A,
                           next_norm=self._next_ln1(layer))
        meta = {"active": act_rows, "n_active": n_active, "checksum": checksum, "k_selected": k_sel,
                "document_tokens": n_doc, "active_rows": A}
        return h_a, A, meta

    def _cacheblend_gradual(self, ids: torch.Tensor, slot: KVSlot, *, prefix_tokens: int, suffix_tokens: int,
                            blend: CacheBlendConfig, global_positions: torch.Tensor | None):
        """CacheBlend with several check layers (``blend.schedule``).

        The first check layer runs as in ``cacheblend``.  Each later check
        layer projects the rows still active (fresh K/V written at their slots,
        deviation partials against the composed cache in the QKV epilogue),
        selects the top ``ratio * N_doc`` active document rows (the active
        list is sorted, so its document rows are a contiguous local range),
        and only those rows attend and continue.
        """
        from ..cacheblend import recompute_count

        cfg, ext = self.cfg, self.ext
        H = cfg.n_kv_heads
        T = ids.numel()
        raw_len = T - suffix_tokens
        n_doc = raw_len - prefix_tokens
        if T > slot.capacity:
            raise ValueError("prompt exceeds slot capacity")
        sched = blend.schedule
        first = sched[0][0]
        if sched[-1][0] >= cfg.n_layers:
            raise ValueError("check_layer lies outside the model")
        n_pre = prefix_tokens if blend.keep_prefix else 0
        h = self.embed(ids)
        rows = self._arange("rows", T)
        gpos = rows if global_positions is None else global_positions
        kpos = global_positions
        for layer in range(first):
            q = self._full_layer(layer, h, slot, gpos, rows, T, kpos)
            self._attn_mlp(layer, h, q, slot, q_rows=None, qpos=gpos, n_keys=T, kpos=kpos, n_rows=T)
        k_sel = recompute_count(n_doc, sched[0][1])
        A = n_pre + k_sel + suffix_tokens
        dev = self.ws.get("dev", (T, 2 * H), torch.float32)
        q = self._full_layer(first, h, slot, gpos, rows, T, kpos, dev, blend.dev_mode)
        active = self._i32("active", T)
        n_active = self._i32("n_active", 1)
        scores = self.ws.get("scores", (max(1, n_doc),), torch.float32)
        ext.cacheblend_select(dev, H, blend.dev_mode, T, prefix_tokens, raw_len, k_sel, blend.keep_prefix, active,
                              n_active, scores, None)
        act = active[:A]
        qpos_a = self._i32("qpos_a", A)
        ext.index_i32(gpos, act, qpos_a)
        h_a = self.ws.get("h_a", (A, cfg.d_model), torch.bfloat16)
        ext.gather_rows(h, act, h_a)
        self._attn_mlp(first, h_a, q, slot, q_rows=act, qpos=qpos_a, n_keys=T, kpos=kpos, n_rows=A)
        later = dict(sched[1:])
        pp = 0
        for layer in range(first + 1, cfg.n_layers):
            if layer not in later:
                qa = self._full_layer(layer, h_a, slot, qpos_a, act, T, kpos)
                self._attn_mlp(layer, h_a, qa, slot, q_rows=None, qpos=qpos_a, n_keys=T, kpos=kpos, n_rows=A)
                continue
            dev2 = self.ws.get("dev_g", (A, 2 * H), torch.float32)
            qa = self._full_layer(layer, h_a, slot, qpos_a, act, T, kpos, dev2, blend.dev_mode)
            k2 = min(recompute_count(n_doc, later[layer]), A - n_pre - suffix_tokens)
            A2 = n_pre + k2 + suffix_tokens
            local = self._i32("g_local", A)
            n_loc = self._i32("g_nloc", 1)
            sc2 = self.ws.get("g_scores", (max(1, A),), torch.float32)
            ext.cacheblend_select(dev2, H, blend.dev_mode, A, n_pre, A - suffix_tokens, k2, blend.keep_prefix,
                                  local, n_loc, sc2, None)
            loc = local[:A2]
            act2 = self._i32(f"g_act{pp}", A2)
            ext.index_i32(act, loc, act2)
            qpos2 = self._i32(f"g_qpos{pp}", A2)
            ext.index_i32(qpos_a, loc, qpos2)
            h2 = self.ws.get(f"g_h{pp}", (A2, cfg.d_model), torch.bfloat16)
            ext.gather_rows(h_a, loc, h2)
            self._attn_mlp(layer, h2, qa, slot, q_rows=loc, qpos=qpos2, n_keys=T, kpos=kpos, n_rows=A2)
            act, qpos_a, h_a, A = act2, qpos2, h2, A2
            pp ^= 1
        meta = {"active": act, "n_active": None, "checksum": None, "k_selected": A - n_pre - suffix_tokens,
                "document_tokens": n_doc, "active_rows": A, "check_layers": [c for c, _ in sched],
                "recompute_ratios": [r for _, r in sched],
                "layer_document_trace": blend.layer_document_trace(cfg.n_layers),
                "layer_document_mean": blend.check_target(cfg.n_layers)}
        return h_a, A, meta

    # ------------------------------------------------------------ decode
    MAX_DECODE_TOKENS = 8192
    MAX_ROWS = 8
    ATTN_SPLIT_ROWS = 512  # query rows up to which prefill attention may split its keys

    def _decode_buffers(self, max_new: int = 0):
        """Fixed-size decode state (captured decode graphs hold these addresses).

        ``pos`` holds the device scalars [rope position, cache slot, virtual
        key count, spare] of the next row; the LM-head kernel advances them.
        """
        if max_new > self.MAX_DECODE_TOKENS:
            raise ValueError(f"max_new_tokens above {self.MAX_DECODE_TOKENS}")
        cfg, ws, R = self.cfg, self.ws, self.MAX_ROWS
        grid = self.ext.gemv_argmax_grid(cfg.vocab)
        if "dec_attn_cnt" not in ws.bufs:  # tickets of the cross-cluster merge: zero between launches
            ws.bufs["dec_attn_cnt"] = torch.zeros(cfg.n_kv_heads * ATTN_CNT_PER_KVH, device=self.device,
                                                  dtype=torch.int32)
        if "dec_pos" not in ws.bufs:
            # pos[3] is a step counter that tensor-parallel ranks turn into flag
            # epochs: it must start equal (zero) on every rank
            ws.bufs["dec_pos"] = torch.zeros(4, device=self.device, dtype=torch.int32)
        return {
            "attn_ws": ws.get("dec_attn_ws", (cfg.n_kv_heads * ATTN_WS_PER_KVH,), torch.float32),
            "attn_cnt": ws.bufs["dec_attn_cnt"],
            "h": ws.get("dec_h", (R, cfg.d_model), torch.bfloat16),
            "q": ws.get("dec_q", (R, cfg.q_size), torch.bfloat16),
            "attn": ws.get("dec_attn", (R, cfg.q_size), torch.bfloat16),
            "act": ws.get("dec_act", (R, cfg.ffn), torch.bfloat16),
            "pos": ws.get("dec_pos", (4,), torch.int32),
            "tok": ws.get("dec_tok", (R,), torch.int32),
            "ids": ws.get("dec_ids", (R,), torch.int32),
            "log": ws.get("dec_log", (self.MAX_DECODE_TOKENS,), torch.int32),
            "gen": ws.get("dec_gen", (1,), torch.int32),
            "pv": ws.get("dec_pv", (R * grid,), torch.float32),
            "pi": ws.get("dec_pi", (R * grid,), torch.int32),
            "counter": ws.get("dec_counter", (1,), torch.int32),
        }

    def _decode_splits(self, capacity: int) -> int:
        """CTAs per kv head (= thread-block cluster size) of the decode attention."""
        return int(self.ext.attention_decode_cluster(capacity, self.cfg.n_kv_heads))

    def _batch_splits(self, capacity: int, n_seq: int, n_kv_heads: int | None = None) -> int:
        """Cluster size of the batched decode attention: the smallest power of two that gives
        every SM a CTA (sequences x kv heads x cluster >= SMs), at most the one-sequence size.
        With 32 sequences of 8 kv heads one CTA per (sequence, kv head) suffices: 66 us per
        layer at 1.7k keys against 206 us with 8-CTA clusters (B200, 0.51 of measured HBM)."""
        kvh = self.cfg.n_kv_heads if n_kv_heads is None else n_kv_heads
        cap = int(self.ext.attention_decode_cluster(capacity, kvh))
        s = 1
        while s < cap and n_seq * kvh * s < self.num_sms:
            s *= 2
        return s

    def set_decode_state(self, *, position: int, slot: int | None = None, n_virtual: int | None = None) -> None:
        """Host-side set of the device scalars (stream-ordered, before a step)."""
        b = self._decode_buffers()
        vals = torch.tensor([position, position if slot is None else slot,
                             (position if n_virtual is None else n_virtual), 0], dtype=torch.int32)
        b["pos"].copy_(vals.pin_memory(), non_blocking=True)

    def first_token(self, hidden_row: torch.Tensor, *, position: int, max_new: int) -> dict:
        """LM head + argmax on the last prompt row; seeds the device-side decode state."""
        b = self._decode_buffers(max_new)
        b["gen"].zero_()
        b["counter"].zero_()
        self.set_decode_state(position=position)
        self.ext.gemv_argmax(hidden_row, self.w.lm_head, self.w.norm, self.cfg.rms_eps, b["pv"], b["pi"],
                             b["counter"], b["tok"], b["log"], b["gen"], self.w.embed, b["h"], None)
        return b

    def _forward_rows(self, slot: KVSlot, b: dict, M: int, splits: int, *, view: torch.Tensor | None,
                      log: bool, feedback: bool, layers=None, key_capacity: int = 0) -> None:
        """One forward of the M rows in b['h'][:M] at the device positions in b['pos'].

        With ``view`` (an int32 slot map of the slot), attention reads the
        virtual key sequence view[0 : pos[2]] and the new rows are written to
        cache slots pos[1].. (RoPE positions pos[0]..); otherwise slot ==
        position and keys are [0, pos[0] + M).
        """
        cfg, ext = self.cfg, self.ext
        H = cfg.n_heads
        h = b["h"][:M]
        pos = b["pos"]
        order = range(len(self.w.layers)) if layers is None else layers
        for layer in order:  # a layer subset (layer-sparse drafting) skips the others as identity
            lw = self.w.layers[layer]
            ext.gemv_qkv(h, lw.w_qkv, lw.ln1, cfg.rms_eps, b["q"][:M], slot.k(layer), slot.v(layer), pos[0:1],
                         self.rope, cfg.n_heads, cfg.n_kv_heads, slot=pos[1:2])
            ext.attention_decode(b["q"][:M], slot.k(layer), slot.v(layer), pos[0:1], H, self.scale, splits,
                                 b["attn"][:M], page_table=view, page_shift=0,
                                 n_virtual=pos[2:3] if view is not None else None, ws=b["attn_ws"],
                                 counters=b["attn_cnt"], l2_prefetch=[lw.w_o, lw.w_gu],
                                 l2_prefetch_bytes=DECODE_L2_PREFETCH, key_capacity=key_capacity)
            ext.gemv_residual(b["attn"][:M], lw.w_o, None, cfg.rms_eps, h, h)
            ext.gemv_swiglu(h, lw.w_gu, lw.ln2, cfg.rms_eps, b["act"][:M])
            ext.gemv_residual(b["act"][:M], lw.w_down, None, cfg.rms_eps, h, h)
        ext.gemv_argmax(h, self.w.lm_head, self.w.norm, cfg.rms_eps, b["pv"], b["pi"], b["counter"], b["tok"],
                        b["log"] if log else None, b["gen"] if log else None,
                        self.w.embed if feedback else None, b["h"][0:1] if feedback else None,
                        pos, 3)

    def decode(self, slot: KVSlot, n_steps: int, *, max_new: int, use_graph: bool = True,
               view: torch.Tensor | None = None, layers: tuple[int, ...] | None = None) -> None:
        """Run ``n_steps`` greedy decode steps from the device state.

        Each step feeds back the previous argmax (its embedding is already in
        h[0]), logs the new token and advances the device scalars.  With a
        ``view`` the steps attend through the slot map (progressive drafting).
        """
        if n_steps <= 0:
            return
        splits = self._decode_splits(slot.capacity)
        b = self._decode_buffers(max_new)
        if not use_graph:
            for _ in range(n_steps):
                self._forward_rows(slot, b, 1, splits, view=view, log=True, feedback=True, layers=layers)
            return
        key = (id(slot), splits, None if view is None else view.data_ptr(), layers)
        graph = self._graphs.get(key)
        if graph is None:
            # one eager step warms up launch attributes; then capture a step
            # against a snapshot of the device state so the real state is
            # only advanced by replays.
            saved = {k: b[k].clone() for k in ("h", "pos", "gen", "log", "tok")}
            self._forward_rows(slot, b, 1, splits, view=view, log=True, feedback=True, layers=layers)
            for k, v in saved.items():
                b[k].copy_(v)
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._forward_rows(slot, b, 1, splits, view=view, log=True, feedback=True, layers=layers)
            for k, v in saved.items():
                b[k].copy_(v)
            self._graphs[key] = graph
        for _ in range(n_steps):
            graph.replay()
        # every replay launches the captured kernels: 5 per layer + LM head
        self.ext.launches += n_steps * (5 * self.cfg.n_layers + 1)

    def verify(self, slot: KVSlot, tokens: torch.Tensor, *, position: int, slot_start: int | None = None,
               view: torch.Tensor | None = None, n_visible: int | None = None, sparse: bool = False) -> torch.Tensor:
        """Batched verifier: forward M <= 8 tokens at positions position.. in one pass.

        Writes their K/V (cache slots slot_start.., default = positions) and
        returns the device int32 argmax prediction after every row (the
        target's next token given the prefix through that row).  With a
        ``view`` the keys are view[0 : n_visible] followed by the M new rows.

        ``sparse`` (views only): size the attention's key split for the view's
        n_visible + M keys instead of the slot's capacity, so a small view of a
        long cache spreads over all CTAs.  The split boundaries then differ
        from those of decoding, so a row's rounding can differ from the
        verifier's: for draft steps, whose tokens are verified afterwards; a
        verification that must equal greedy decoding keeps the default.
        """
        M = int(tokens.numel())
        if not 1 <= M <= self.MAX_ROWS:
            raise ValueError("verify handles 1..8 tokens")
        if sparse and view is None:
            raise ValueError("sparse applies to verification over a view")
        b = self._decode_buffers()
        nv = None if view is None else int(n_visible) + M
        key_cap = nv if sparse else 0
        splits = self._decode_splits(key_cap if sparse else slot.capacity)
        b["ids"][:M].copy_(tokens.to(torch.int32), non_blocking=True)
        self.ext.embedding(b["ids"][:M], self.w.embed, b["h"][:M])
        self.set_decode_state(position=position, slot=slot_start, n_virtual=nv)
        self._forward_rows(slot, b, M, splits, view=view, log=False, feedback=False, key_capacity=key_cap)
        return b["tok"][:M]

    def generated_tokens(self, max_new: int) -> torch.Tensor:
        """Device view of the token log (first ``max_new`` entries)."""
        return self._decode_buffers(max_new)["log"][:max_new]

    # ------------------------------------------------------ batched decode
    MAX_BATCH = 32  # sequences per batched step (the skinny tensor-core GEMM takes 32 rows)

    def batch_slots(self, n_seq: int, capacity: int) -> list[KVSlot]:
        """``n_seq`` serving slots back to back in one buffer (a batched step addresses them by stride)."""
        if not 1 <= n_seq <= self.MAX_BATCH:
            raise ValueError(f"1..{self.MAX_BATCH} sequences per batched step")
        per = KVSlot.nbytes_for(self.cfg, capacity) // 2
        buf = torch.empty(n_seq * per, dtype=torch.bfloat16, device=self.device)
        return [KVSlot.from_buffer(self.cfg, capacity, buf[i * per:(i + 1) * per]) for i in range(n_seq)]

    def _batch_buffers(self) -> dict:
        cfg, ws, B = self.cfg, self.ws, self.MAX_BATCH
        if "bt_gen" not in ws.bufs:
            ws.bufs["bt_gen"] = torch.zeros(1, device=self.device, dtype=torch.int64)
        if "bt_skinny_ws" not in ws.bufs:
            w0 = self.w.layers[0]
            shapes = [tuple(w0.w_qkv.shape), tuple(w0.w_o.shape), tuple(w0.w_gu.shape), tuple(w0.w_down.shape),
                      tuple(self.w.lm_head.shape)]
            need = max(int(self.ext.skinny_splits(n, k)) * n * 32 for n, k in shapes)
            ws.bufs["bt_skinny_ws"] = torch.empty(need, device=self.device, dtype=torch.float32)
        return {"h": ws.get("bt_h", (B, cfg.d_model), torch.bfloat16),
                "x": ws.get("bt_x", (B, cfg.d_model), torch.bfloat16),
                "q": ws.get("bt_q", (B, cfg.q_size), torch.bfloat16),
                "attn": ws.get("bt_attn", (B, cfg.q_size), torch.bfloat16),
                "act": ws.get("bt_act", (B, cfg.ffn), torch.bfloat16),
                "logits": ws.get("bt_logits", (B, cfg.vocab), torch.bfloat16),
                "tok": ws.get("bt_tok", (B,), torch.int32),
                "pos": ws.get("bt_pos", (B,), torch.int32),
                "gen": ws.bufs["bt_gen"],
                "log": ws.get("bt_log", (self.MAX_DECODE_TOKENS, B), torch.int32),
                "skinny_ws": ws.bufs["bt_skinny_ws"]}

    def batch_first_tokens(self, last_rows: torch.Tensor) -> torch.Tensor:
        """Greedy first token of each sequence from its last prompt row (pre-norm hidden, [B, d]):
        final RMSNorm, LM head on the tensor cores, row argmax.  Returns the device int32 [B]."""
        B = last_rows.shape[0]
        bb = self._batch_buffers()
        x = bb["x"][:B]
        self.ext.rmsnorm(last_rows, None, self.w.norm, self.cfg.rms_eps, x)
        self.ext.skinny_gemm(x, self.w.lm_head, 0, bb["logits"][:B], None, bb["skinny_ws"])
        self.ext.row_argmax(bb["logits"][:B], bb["tok"])
        return bb["tok"][:B]

    def start_batch(self, slots: list[KVSlot], first_tokens: torch.Tensor, positions, *, max_new: int) -> None:
        """Seed a batched greedy decode: sequence b produced ``first_tokens[b]`` (device int32) at
        position ``positions[b]`` (its prompt length)."""
        B = len(slots)
        if first_tokens.numel() != B or len(positions) != B:
            raise ValueError("one first token and one position per sequence")
        bb = self._batch_buffers()
        if max_new > bb["log"].shape[0]:
            raise ValueError("max_new exceeds the batched token log")
        bb["tok"][:B].copy_(first_tokens.to(torch.int32), non_blocking=True)
        bb["pos"][:B].copy_(torch.as_tensor(list(positions), dtype=torch.int32).pin_memory(), non_blocking=True)
        bb["log"][0, :B].copy_(bb["tok"][:B])
        bb["gen"].fill_(1)
        self.ext.embedding(bb["tok"][:B], self.w.embed, bb["h"][:B])

    def _batch_step(self, slots: list[KVSlot], splits: int) -> None:
        """One greedy step of every sequence: row b is sequence b at its own position and slot."""
        cfg, ext = self.cfg, self.ext
        B = len(slots)
        bb = self._batch_buffers()
        h, x, pos_rows, ws = bb["h"][:B], bb["x"][:B], bb["pos"][:B], bb["skinny_ws"]
        stride = (slots[1].data.data_ptr() - slots[0].data.data_ptr()) // 2 if B > 1 else 0
        for layer, lw in enumerate(self.w.layers):
            ext.rmsnorm(h, None, lw.ln1, cfg.rms_eps, x)
            ext.skinny_qkv(x, lw.w_qkv, bb["q"][:B], slots[0].k(layer), slots[0].v(layer), pos_rows, self.rope,
                           cfg.n_heads, cfg.n_kv_heads, ws, pos_rows=pos_rows, seq_stride=stride)
            ext.attention_decode(bb["q"][:B], slots[0].k(layer), slots[0].v(layer), pos_rows, cfg.n_heads,
                                 self.scale, splits, bb["attn"][:B], pos_rows=pos_rows, seq_stride=stride,
                                 l2_prefetch=[lw.w_o, lw.w_gu], l2_prefetch_bytes=BATCH_L2_PREFETCH)
            ext.skinny_gemm(bb["attn"][:B], lw.w_o, 1, h, h, ws)
            ext.rmsnorm(h, None, lw.ln2, cfg.rms_eps, x)
            ext.skinny_gemm(x, lw.w_gu, 2, bb["act"][:B], None, ws)
            ext.skinny_gemm(bb["act"][:B], lw.w_down, 1, h, h, ws)
        ext.rmsnorm(h, None, self.w.norm, cfg.rms_eps, x)
        ext.skinny_gemm(x, self.w.lm_head, 0, bb["logits"][:B], None, ws)
        ext.row_argmax(bb["logits"][:B], bb["tok"])
        bb["log"][:, :B].index_copy_(0, bb["gen"], bb["tok"][:B].view(1, B))
        bb["gen"].add_(1)
        pos_rows.add_(1)
        ext.embedding(bb["tok"][:B], self.w.embed, h)

    def decode_batch(self, slots: list[KVSlot], n_steps: int, *, use_graph: bool = True) -> None:
        """``n_steps`` batched greedy steps from the state ``start_batch`` (or earlier steps) left."""
        if n_steps <= 0:
            return
        if len({s.capacity for s in slots}) != 1:
            raise ValueError("batched slots share one capacity")
        splits = self._batch_splits(slots[0].capacity, len(slots))
        if not use_graph:
            for _ in range(n_steps):
                self._batch_step(slots, splits)
            return
        key = ("batch", tuple(id(s) for s in slots), splits)
        graph = self._graphs.get(key)
        if graph is None:
            bb = self._batch_buffers()
            saved = {k: bb[k].clone() for k in ("h", "tok", "pos", "gen", "log")}
            self._batch_step(slots, splits)  # warm step, then capture against the saved state
            for k, v in saved.items():
                bb[k].copy_(v)
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._batch_step(slots, splits)
            for k, v in saved.items():
                bb[k].copy_(v)
            self._graphs[key] = graph
        for _ in range(n_steps):
            graph.replay()
        # per layer: 2 norms, QKV (GEMM + reduce), attention, 3 skinny GEMMs (GEMM + reduce each)
        self.ext.launches += n_steps * (11 * self.cfg.n_layers + 7)

    def batch_tokens(self, n_seq: int, n_tokens: int) -> torch.Tensor:
        """Device view of the batched token log: [n_tokens, n_seq] (column b = sequence b)."""
        return self._batch_buffers()["log"][:n_tokens, :n_seq]

    def release_graphs(self) -> None:
        self._graphs.clear()
