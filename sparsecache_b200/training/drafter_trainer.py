"""Sparse-KV EAGLE drafter training on B200: batched, graph-captured, data parallel.

Parity with the reference trainer experiments/train_sparse_kv_eagle.py:
the same model construction (``build_model`` :57-94: EAGLE trunk frozen in
bf16, the sparse-memory adapter kept as fp32 master weights), the same
losses (compressed-vocabulary distillation, optional cosine feature loss,
a margin contrast against another request's memory and a "base contrast"
against the memory-disabled model, :97-175 and :571-640), trainability
switches (``configure_trainable_modules`` :189-205), adapter checkpoints
(``build_adapter_checkpoint`` / ``load_adapter_checkpoint`` :208-265,
format ``sparsecache.sparse-kv-eagle-adapter.v2``) and the evaluation
(teacher-forced top-1 over 8 tokens and the accepted prefix of greedy
drafts, under exact / zero / shuffled / disabled memory, :268-381).

What is different is how a step runs:
  * a step trains ``global_batch`` sequences at once (the reference trains
    one at a time): the positive and the contrast rows run as one batched
    recurrence of 2B rows, each row with its own sparse memory view read in
    place from the HBM-resident teacher bank by the K13 kernel;
  * all trainable parameters are views into one flat fp32 buffer and their
    gradients accumulate into one flat fp32 buffer, so the optimizer is one
    fused AdamW kernel pair (global-norm clip + update, step count and
    learning rate on the device) instead of per-tensor launches;
  * the adapter's memory projections form their weight gradients after the
    recurrence, one tensor-core GEMM per weight over all positions with fp32
    sums (``deferred_grad.py``), instead of 256 per-position products;
  * with several GPUs the flat gradient/parameter buffers are CUDA-IPC peer
    memory: each rank sums its 1/N shard of every peer's gradients in rank
    order, bucket by bucket as the backward finishes them (everything
    autograd wrote, then each deferred weight right after its GEMM, on a
    side stream while the next GEMM runs), all ranks agree on the clip
    coefficient, each rank runs AdamW on its shard (ZeRO-1 optimizer state)
    and stores the result straight into every peer's parameter buffer; flags
    with bounded waits order the phases.  No NCCL call is on the step path;
  * the whole step (gather of the batch from the bank, recurrent forward,
    loss, backward, optimizer, DP exchange) is captured once as a CUDA graph
    and replayed; the host only writes the next batch's indices;
  * the trunk's self-attention runs forward and backward on the K14 kernels
    (``ops.linear.recurrent_attention``), the LM head through the fused
    LM-head/log-sum-exp kernels, the memory attention through K13; the frozen
    projections can run on the tensor-core GEMMs (``tc_linears``).
"""
from __future__ import annotations

import json
import math
import os
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..models.sparse_kv_draft import accepted_prefix_length
from ..models.sparse_kv_eagle import SparseKVEagleConfig, SparseKVEagleDrafter
from ..ops.sparse_attention import MemoryBatch
from .losses import (compressed_distillation_from_lse, compressed_distillation_loss, compressed_id_table,
                     compressed_target_score, compressed_target_score_from_lse, feature_distillation_loss)
from .teacher import DeviceTeacherBank, pick_mismatched

ADAPTER_FORMAT = "sparsecache.sparse-kv-eagle-adapter.v2"
TIMEOUT_NS = 20_000_000_000


@dataclass
class DrafterTrainConfig:
    lr: float = 1e-4
    weight_decay: float = 0.01
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    grad_clip: float = 1.0
    prefix_decay: float = 0.9
    hard_weight: float = 1.0
    soft_weight: float = 0.5
    contrast_weight: float = 0.5
    contrast_margin: float = 0.25
    base_contrast_weight: float = 0.25
    feature_weight: float = 0.0
    global_batch: int = 32
    window_tokens: int = 0  # 0: the whole teacher horizon
    use_graph: bool = True
    # frozen trunk projections forward/backward on this package's tensor-core GEMMs; off by
    # default: at 64 rows per recurrent position the library's single-kernel small GEMMs are
    # faster (8B width, B200: 570 vs 484 ms per step), see ops/linear.py
    tc_linears: bool = False
    # the adapter's memory projections form their weight gradients after the recurrence, one
    # tensor-core GEMM per weight (fp32 sums over all positions); with data parallelism each
    # finished weight's reduce-scatter overlaps the next weight's GEMM (training/deferred_grad.py)
    defer_weight_grads: bool = True
    # with several GPUs: reduce each gradient bucket as soon as it is final (False: one
    # reduce-scatter of the whole buffer after the backward, the A/B control)
    overlap_exchange: bool = True
    # with several GPUs: the NCCL control instead of the peer-memory exchange (every rank keeps
    # the whole buffer, ncclAllReduce of the flat gradient after the backward, AdamW everywhere)
    nccl_exchange: bool = False
    seed: int = 0

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


# ------------------------------------------------------------ model helpers
def configure_trainable_modules(model: SparseKVEagleDrafter, *, train_fc: bool, train_midlayer: bool,
                                adapter_scale_init: float) -> None:
    """Open the requested EAGLE modules (as fp32 master weights) and set the adapter scale."""
    model.adapter_scale.data.fill_(adapter_scale_init)
    for flag, module in ((train_fc, model.fc), (train_midlayer, model.midlayer)):
        if flag:
            module.float()
            for p in module.parameters():
                p.requires_grad_(True)


def prepare_for_training(model: SparseKVEagleDrafter, device) -> SparseKVEagleDrafter:
    """Trunk in bf16, sparse-memory adapter (and anything trainable) in fp32."""
    model.to(device=device)
    for module in (model.midlayer, model.fc, model.norm, model.lm_head):
        if not any(p.requires_grad for p in module.parameters()):
            module.to(torch.bfloat16)
    for module in (model.memory_norm, model.memory_attention, model.stage_layer_bias, model.memory_gate,
                   model.memory_delta):
        module.float()
    model.adapter_scale.data = model.adapter_scale.data.float()
    return model


def build_adapter_checkpoint(model: SparseKVEagleDrafter, *, completed_steps: int, training_args: dict,
                             extra: dict | None = None) -> dict[str, Any]:
    out = {
        "format": ADAPTER_FORMAT,
        "created_at_ns": time.time_ns(),
        "config": model.config.to_dict(),
        "adapter_state_dict": model.adapter_state_dict(),
        "trainable_parameter_names": [n for n, p in model.named_parameters() if p.requires_grad],
        "completed_steps": completed_steps,
        "training_args": training_args,
    }
    out.update(extra or {})
    return out


def load_adapter_checkpoint(model: SparseKVEagleDrafter, checkpoint_path: Path | str) -> dict[str, Any]:
    """Load adapter weights (shape-checked, unknown names refused); trainability is unchanged."""
    ckpt = torch.load(checkpoint_path, map_location="cpu", weights_only=True)
    state = ckpt.get("adapter_state_dict")
    if not isinstance(state, dict) or not state:
        raise ValueError("resume checkpoint has no adapter_state_dict")
    model_state = model.state_dict()
    unknown = set(state) - set(model_state)
    if unknown:
        raise ValueError(f"resume checkpoint has unknown tensors: {sorted(unknown)}")
    bad = {n: (tuple(t.shape), tuple(model_state[n].shape)) for n, t in state.items()
           if t.shape != model_state[n].shape}
    if bad:
        raise ValueError(f"resume checkpoint tensor shapes differ: {bad}")
    model.load_state_dict(state, strict=False)
    return ckpt


# ------------------------------------------------------------ flat buffers
class FlatTrainables:
    """Trainable parameters as views of one flat fp32 buffer, gradients likewise.

    ``alloc(numel)`` returns the backing fp32 tensors (plain device memory, or
    CUDA-IPC shared memory for data parallelism).  The length is padded to a
    multiple of ``4 * world`` so every rank's shard starts 16-byte aligned.
    """

    def __init__(self, params: Sequence[nn.Parameter], *, world: int = 1, alloc=None, device=None) -> None:
        self.params = list(params)
        if not self.params:
            raise ValueError("nothing to train")
        n = sum(p.numel() for p in self.params)
        q = 4 * world
        self.numel = n
        self.padded = -(-n // q) * q
        dev = device if device is not None else self.params[0].device
        alloc = alloc or (lambda m: torch.zeros(m, device=dev, dtype=torch.float32))
        self.param = alloc(self.padded)
        self.grad = alloc(self.padded)
        self.grad.zero_()
        self.offsets: dict[int, tuple[int, int]] = {}  # id(param) -> (offset, numel)
        off = 0
        for p in self.params:
            k = p.numel()
            view = self.param[off:off + k].view_as(p)
            view.copy_(p.detach().float())
            p.data = view
            p.grad = self.grad[off:off + k].view_as(p)
            self.offsets[id(p)] = (off, k)
            off += k

    def shard(self, world: int) -> int:
        return self.padded // world

    def buckets(self, late: Sequence[nn.Parameter]) -> list[list[tuple[int, int]]]:
        """Flat ranges of the exchange buckets: everything but ``late`` first, then each of ``late``.

        Bucket 0 (gradients final when autograd's backward returns) is the
        complement of the late parameters' ranges within the padded buffer;
        bucket 1 + i is the range of ``late[i]``.
        """
        spans = sorted(self.offsets[id(p)] for p in late)
        rest, cur = [], 0
        for off, k in spans:
            if off > cur:
                rest.append((cur, off))
            cur = off + k
        if cur < self.padded:
            rest.append((cur, self.padded))
        out = [rest]
        for p in late:
            off, k = self.offsets[id(p)]
            out.append([(off, off + k)])
        return out


class FusedAdamW:
    """Device-side AdamW over a FlatTrainables set (1 GPU, or a DP rank's shard)."""

    def __init__(self, flat: FlatTrainables, cfg: DrafterTrainConfig, *, shard: int | None = None) -> None:
        dev = flat.param.device
        n = shard if shard is not None else flat.padded
        self.exp_avg = torch.zeros(n, device=dev, dtype=torch.float32)
        self.exp_avg_sq = torch.zeros(n, device=dev, dtype=torch.float32)
        self.hyper = torch.tensor([cfg.lr, cfg.beta1, cfg.beta2, cfg.eps, cfg.weight_decay, cfg.grad_clip, 0.0, 0.0],
                                  device=dev, dtype=torch.float32)
        self.state = torch.zeros(8, device=dev, dtype=torch.float32)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 1
        self.partial = torch.zeros(2 * sms, device=dev, dtype=torch.float32)
        self.counter = torch.zeros(1, device=dev, dtype=torch.int32)
        self.flat = flat

    def step(self) -> None:
        if self.flat.param.device.type == "cpu":  # host oracle of the kernel pair (CPU tests only)
            self._step_reference()
            return
        ops.ext().adamw_step(self.flat.param, self.flat.grad, self.exp_avg, self.exp_avg_sq, self.hyper, self.state,
                             self.partial, self.counter)

    @torch.no_grad()
    def _step_reference(self) -> None:
        lr, b1, b2, eps, wd, max_norm = self.hyper.tolist()[:6]
        g = self.flat.grad
        norm = float(g.double().square().sum().sqrt())
        coef = min(1.0, max_norm / (norm + 1e-6)) if max_norm > 0 else 1.0
        step = float(self.state[0]) + 1.0
        bc1, bc2 = 1.0 - b1 ** step, 1.0 - b2 ** step
        self.state[:5] = torch.tensor([step, bc1, bc2, norm, coef])
        gc = g * coef
        p = self.flat.param
        p.mul_(1.0 - lr * wd)
        self.exp_avg.lerp_(gc, 1.0 - b1)
        self.exp_avg_sq.mul_(b2).addcmul_(gc, gc, value=1.0 - b2)
        p.addcdiv_(self.exp_avg, self.exp_avg_sq.sqrt() / math.sqrt(bc2) + eps, value=-lr / bc1)

    def set_lr(self, lr: float) -> None:
        self.hyper[0].fill_(lr)

    def state_dict(self) -> dict[str, torch.Tensor]:
        return {"exp_avg": self.exp_avg.cpu(), "exp_avg_sq": self.exp_avg_sq.cpu(), "state": self.state.cpu()}

    def load_state_dict(self, sd: dict[str, torch.Tensor]) -> None:
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        self.state.copy_(sd["state"])


class DataParallelAdamW(FusedAdamW):
    """Reduce-scatter + AdamW + all-gather over peer memory (see module docstring)."""

    def __init__(self, flat: FlatTrainables, cfg: DrafterTrainConfig, group, param_ptrs, grad_ptrs) -> None:
        self.world, self.rank = group.size, group.rank
        super().__init__(flat, cfg, shard=flat.shard(self.world))
        self.group = group
        dev = flat.param.device
        self.red_grad = torch.zeros(flat.shard(self.world), device=dev, dtype=torch.float32)
        self.param_ptrs, self.grad_ptrs = param_ptrs, grad_ptrs
        w = self.world
        self.norm_buf, norm_ptrs = group.shared(4 * max(w, 4))
        self.norm_ptrs = norm_ptrs
        self.flag_buf, flag_ptrs = group.shared(4 * 3 * 8)
        self.flags = self.flag_buf.view(torch.int32)
        self.flag_ptrs = flag_ptrs
        self.epoch = torch.zeros(1, device=dev, dtype=torch.int32)
        self.status = torch.zeros(1, device=dev, dtype=torch.int32)
        self.buckets: list[list[tuple[int, int]]] | None = None

    def _peer_flag(self, kind: int, peer: int) -> int:
        # flag block of ``peer``: [kind][source rank]
        return self.flag_ptrs[peer] + 4 * (kind * 8 + self.rank)

    # -------------------------------------------- reduce-scatter overlapped with the backward
    def enable_buckets(self, buckets: list[list[tuple[int, int]]], *, grid: int | None = None) -> None:
        """Reduce the gradient bucket by bucket as the backward finishes them.

        ``buckets[b]`` lists flat ranges.  Each rank releases bucket b's flag
        in every peer once its own gradients of the bucket are final
        (``bucket_ready``); a side stream then waits (bounded) for every
        rank's release and sums this rank's shard of the bucket, while the
        main stream goes on with the backward.  ``grid`` CTAs per bucket
        kernel (default 2 per SM: the reduction is NVLink- and HBM-bound, and
        32 CTAs measured slower than no overlap at all).
        """
        nb = len(buckets)
        self.buckets = buckets
        self.bucket_buf, self.bucket_ptrs = self.group.shared(4 * 8 * nb)
        self.bucket_flags = self.bucket_buf.view(torch.int32).view(nb, 8)
        self.comm = torch.cuda.Stream(self.flat.param.device)
        if grid is None:  # 2 CTAs per SM; SC_DP_BUCKET_GRID overrides (A/B runs)
            sms = torch.cuda.get_device_properties(self.flat.param.device).multi_processor_count
            grid = int(os.environ.get("SC_DP_BUCKET_GRID", str(2 * sms)))
        self.reduce_grid = max(1, min(1024, grid))

    def bucket_ready(self, b: int) -> None:
        x = ops.ext()
        main = torch.cuda.current_stream()
        x.signal_epoch([self.bucket_ptrs[p] + 4 * (b * 8 + self.rank) for p in range(self.world)], self.epoch, 0)
        self.comm.wait_stream(main)
        with torch.cuda.stream(self.comm):
            for lo, hi in self.buckets[b]:
                x.dp_reduce_range(self.world, self.rank, self.flat.padded, self.flat.shard(self.world),
                                  self.grad_ptrs, self.bucket_flags[b], self.epoch, lo, hi, TIMEOUT_NS,
                                  self.status, self.red_grad, self.reduce_grid)

    def step_reduced(self) -> None:
        """Clip + AdamW + all-gather after every bucket was reduced (joins the side stream)."""
        torch.cuda.current_stream().wait_stream(self.comm)
        self._dp_step(pre_reduced=True)

    def begin_step(self) -> None:
        """Advance the device epoch and wait until every rank's last update landed here."""
        x = ops.ext()
        x.bump_counter(self.epoch)
        x.wait_all(self.flags[16:24], self.world, self.epoch, -1, TIMEOUT_NS, self.status)

    def step(self) -> None:
        """Reduce-scatter of the whole gradient, clip, AdamW, all-gather (after the backward)."""
        ops.ext().signal_epoch([self._peer_flag(0, p) for p in range(self.world)], self.epoch, 0)
        self._dp_step(pre_reduced=False)

    def _dp_step(self, *, pre_reduced: bool) -> None:
        ops.ext().dp_adamw_step(
            self.world, self.rank, self.flat.padded, self.flat.shard(self.world), self.grad_ptrs, self.param_ptrs,
            self.norm_ptrs, self.flags[0:8], self.flags[8:16], [self._peer_flag(1, p) for p in range(self.world)],
            [self._peer_flag(2, p) for p in range(self.world)], self.epoch, TIMEOUT_NS, self.status, self.red_grad,
            self.exp_avg, self.exp_avg_sq, self.hyper, self.state, self.partial, self.counter,
            pre_reduced=pre_reduced)

    def check(self) -> None:
        code = int(self.status.item())
        if code:
            raise RuntimeError(f"data-parallel optimizer timed out waiting for a peer (status {code})")


class _DPGroup:
    """IPC-shared allocation over a torch.distributed group (one process per GPU)."""

    def __init__(self) -> None:
        import torch.distributed as dist

        self.rank = dist.get_rank()
        self.size = dist.get_world_size()
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._opened: list[int] = []
        self._keep: list[torch.Tensor] = []

    def shared(self, nbytes: int):
        import torch.distributed as dist

        x = ops.ext()
        buf, handle = x.shared_empty(int(nbytes), self.device.index)
        self._keep.append(buf)
        handles = [None] * self.size
        dist.all_gather_object(handles, handle)
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(buf.data_ptr())
            else:
                p = x.shared_open(h)
                self._opened.append(p)
                ptrs.append(p)
        return buf, ptrs

    def close(self) -> None:
        x = ops.ext()
        for p in self._opened:
            x.shared_close(p)
        self._opened.clear()


# ------------------------------------------------------------------ trainer
class EagleDrafterTrainer:
    """Training loop of a ``SparseKVEagleDrafter`` over a ``DeviceTeacherBank``."""

    def __init__(self, model: SparseKVEagleDrafter, bank: DeviceTeacherBank, rope_cos: torch.Tensor,
                 rope_sin: torch.Tensor, cfg: DrafterTrainConfig, *, distributed: bool = False) -> None:
        import torch.distributed as dist

        self.model, self.bank, self.cfg = model, bank, cfg
        self.device = bank.input_ids.device
        self.rope_cos = rope_cos.to(self.device, torch.bfloat16)  # [positions, D]
        self.rope_sin = rope_sin.to(self.device, torch.bfloat16)
        self.world = dist.get_world_size() if distributed else 1
        self.rank = dist.get_rank() if distributed else 0
        if cfg.global_batch % self.world:
            raise ValueError("the global batch must divide evenly over the ranks")
        self.local_batch = cfg.global_batch // self.world
        self.horizon = bank.horizon if cfg.window_tokens <= 0 else min(cfg.window_tokens, bank.horizon)
        self.stash = None
        if cfg.defer_weight_grads:
            from .deferred_grad import defer_adapter_linears

            self.stash = defer_adapter_linears(model, self.device)
        params = model.adapter_parameters()
        self.group = None
        self.nccl = distributed and cfg.nccl_exchange
        if self.nccl:
            self.flat = FlatTrainables(params, device=self.device)
            dist.broadcast(self.flat.param, src=0)
            self.opt = FusedAdamW(self.flat, cfg)
        elif distributed:
            self.group = _DPGroup()
            n = sum(p.numel() for p in params)
            padded = -(-n // (4 * self.world)) * (4 * self.world)
            pbuf, pptrs = self.group.shared(4 * padded)
            gbuf, gptrs = self.group.shared(4 * padded)
            bufs = iter((pbuf.view(torch.float32), gbuf.view(torch.float32)))
            self.flat = FlatTrainables(params, world=self.world, alloc=lambda m: next(bufs)[:m])
            dist.broadcast(self.flat.param, src=0)  # identical start on every rank
            self.opt = DataParallelAdamW(self.flat, cfg, self.group, pptrs, gptrs)
            if self.stash is not None and cfg.overlap_exchange:
                self.opt.enable_buckets(self.flat.buckets([lin.weight for lin in self.stash.linears]))
            torch.cuda.synchronize(self.device)
            dist.barrier()
        else:
            self.flat = FlatTrainables(params, device=self.device)
            self.opt = FusedAdamW(self.flat, cfg)
        B = self.local_batch
        self.idx = torch.zeros(B, device=self.device, dtype=torch.int64)
        self.neg = torch.zeros(B, device=self.device, dtype=torch.int64)
        self.loss = torch.zeros((), device=self.device)
        self.components = {k: torch.zeros((), device=self.device) for k in
                           ("hard_loss", "soft_loss", "label_coverage", "topk_coverage", "contrast_loss",
                            "base_contrast_loss", "feature_loss")}
        self.steps_done = 0
        self._graph = None
        self._pinned = torch.empty(2 * B, dtype=torch.int64)
        if self.device.type == "cuda":
            self._pinned = self._pinned.pin_memory()
        self.launches_per_step: int | None = None
        # frozen trunk projections (fc, q/k/v/o, gate/up/down) on this package's GEMM, fwd + dX
        self.tc_linears: list[str] = []
        if cfg.tc_linears and self.device.type == "cuda" and ops.available():
            from ..ops.linear import use_tc_for_frozen_linears

            self.tc_linears = use_tc_for_frozen_linears(model)
        # frozen LM head: logits go through the fused log-sum-exp / gather path
        # (no fp32 [rows, vocab] tensors); a trainable head keeps plain logits
        self.head = None
        if not model.lm_head.weight.requires_grad:
            from ..ops.lm_loss import FrozenLMHead

            self.head = FrozenLMHead(model.lm_head.weight)

    # ------------------------------------------------------------ batching
    def batch_indices(self, step: int) -> tuple[list[int], list[int]]:
        """Sequences of ``step`` for this rank (disjoint across ranks) and their contrast partners."""
        S, G, B = self.bank.size, self.cfg.global_batch, self.local_batch
        pos = [(step * G + self.rank * B + i) % S for i in range(B)]
        groups = self.bank.groups or list(range(S))
        neg = [pick_mismatched(groups, p) for p in pos]
        return pos, neg

    def _positions(self, rows: torch.Tensor, t: int):
        pos = self.bank.prompt_tokens.index_select(0, rows)[:, None] + torch.arange(t, device=self.device)
        return self.rope_cos[pos], self.rope_sin[pos]  # [B, t, D]

    # ------------------------------------------------------------ step body
    def _body(self) -> None:
        cfg, bank, model = self.cfg, self.bank, self.model
        if self.world > 1 and not self.nccl:
            self.opt.begin_step()
        self.flat.grad.zero_()
        t = self.horizon
        idx, neg = self.idx, self.neg
        ids = bank.input_ids.index_select(0, idx)[:, :t]
        labels = bank.labels.index_select(0, idx)[:, :t]
        top_ids = bank.topk_ids.index_select(0, idx)[:, :t]
        top_lp = bank.topk_logprobs.index_select(0, idx)[:, :t]
        seeds = bank.seed_hidden.index_select(0, idx).to(model.fc.weight.dtype)
        cos, sin = self._positions(idx, t)
        stage = bank.stage(idx)
        rows = torch.cat((idx, neg)).to(torch.int32)
        mem = MemoryBatch(bank.mem_k, bank.mem_v, bank.idx, bank.n_vis, rows)
        two = lambda x: torch.cat((x, x))  # noqa: E731  (the contrast rows reuse the inputs)
        B = idx.shape[0]
        if self.stash is not None:
            self.stash.begin(2 * B, t)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=self.device.type == "cuda"):
            feats = model.recurrent_forward(two(ids), two(seeds), mem, None, two(cos), two(sin), two(stage))
            if self.head is not None:
                # positive rows: label + teacher top-k; contrast rows: label only (-1 padded)
                table = compressed_id_table(model, labels, top_ids)
                neg_table = torch.full_like(table, -1)
                neg_table[..., 0] = table[..., 0]
                t_all = torch.cat((table, neg_table))
                lse, z = self.head.lse_gather(feats.reshape(-1, feats.shape[-1]), t_all.reshape(2 * B * t, -1))
                lse, z = lse.view(2 * B, t), z.view(2 * B, t, -1)
                loss, comps = compressed_distillation_from_lse(
                    lse[:B], z[:B], table, top_lp, prefix_decay=cfg.prefix_decay, hard_weight=cfg.hard_weight,
                    soft_weight=cfg.soft_weight, check_coverage=False)
                pos_score = compressed_target_score_from_lse(lse[:B], z[:B, :, 0], table[..., 0],
                                                             prefix_decay=cfg.prefix_decay)
                neg_score = compressed_target_score_from_lse(lse[B:], z[B:, :, 0], table[..., 0],
                                                             prefix_decay=cfg.prefix_decay)
            else:
                logits = model.lm_head(feats)
                pos_logits, neg_logits = logits[:B], logits[B:]
                loss, comps = compressed_distillation_loss(
                    model, pos_logits, labels, top_ids, top_lp, prefix_decay=cfg.prefix_decay,
                    hard_weight=cfg.hard_weight, soft_weight=cfg.soft_weight, check_coverage=False)
                pos_score = compressed_target_score(model, pos_logits, labels, prefix_decay=cfg.prefix_decay)
                neg_score = compressed_target_score(model, neg_logits, labels, prefix_decay=cfg.prefix_decay)
            if cfg.feature_weight > 0.0:
                if bank.teacher_hidden is None:
                    raise ValueError("feature loss requires teacher hidden states")
                th = bank.teacher_hidden.index_select(0, idx)[:, :t]
                f_loss = feature_distillation_loss(feats[:B], th, prefix_decay=cfg.prefix_decay)
                loss = loss + cfg.feature_weight * f_loss
                comps["feature_loss"] = f_loss.detach()
            contrast = F.relu(cfg.contrast_margin - pos_score + neg_score).mean()
            with torch.no_grad():
                base_feats = model.recurrent_forward(ids, seeds, None, None, cos, sin, stage, use_memory=False)
                if self.head is not None:
                    d_lab = model.draft_ids(labels)
                    b_lse, b_z = self.head.lse_gather(base_feats.reshape(-1, base_feats.shape[-1]),
                                                      d_lab.reshape(-1, 1))
                    base_score = compressed_target_score_from_lse(b_lse.view(B, t), b_z.view(B, t), d_lab,
                                                                  prefix_decay=cfg.prefix_decay)
                else:
                    base_score = compressed_target_score(model, model.lm_head(base_feats), labels,
                                                         prefix_decay=cfg.prefix_decay)
            base_contrast = F.relu(cfg.contrast_margin / 2 - pos_score + base_score).mean()
            loss = loss + cfg.contrast_weight * contrast + cfg.base_contrast_weight * base_contrast
        loss.backward()
        if self.nccl:  # control: one NCCL all-reduce (mean) of the whole gradient, then AdamW on every rank
            import torch.distributed as dist

            if self.stash is not None:
                self.stash.finish()
            dist.all_reduce(self.flat.grad, op=dist.ReduceOp.AVG)
            self.opt.step()
        elif self.stash is None:
            self.opt.step()
        elif self.world > 1 and self.cfg.overlap_exchange:
            # bucket 0 (every gradient autograd wrote) is final now; each deferred weight is
            # final after its GEMM: its reduce-scatter runs on the side stream during the next GEMM
            self.opt.bucket_ready(0)
            self.stash.finish(on_weight=lambda k: self.opt.bucket_ready(1 + k))
            self.opt.step_reduced()
        else:
            self.stash.finish()
            self.opt.step()
        self.loss.copy_(loss.detach())
        comps["contrast_loss"] = contrast.detach()
        comps["base_contrast_loss"] = base_contrast.detach()
        for k, v in comps.items():
            self.components[k].copy_(v)

    def _write_batch(self, step: int) -> None:
        pos, neg = self.batch_indices(step)
        B = self.local_batch
        self._pinned[:B] = torch.tensor(pos)
        self._pinned[B:] = torch.tensor(neg)
        self.idx.copy_(self._pinned[:B], non_blocking=True)
        self.neg.copy_(self._pinned[B:], non_blocking=True)

    def warmup_and_capture(self, warmup: int = 3) -> None:
        """Eager warm-up steps (real updates), then capture one step as a CUDA graph."""
        if self.device.type != "cuda":
            for _ in range(warmup):
                self.train_step()
            return
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._write_batch(self.steps_done)
                self._body()
                self.steps_done += 1
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        if not self.cfg.use_graph:
            return
        self._write_batch(self.steps_done)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._body()
        self._graph = g  # capturing executed nothing: the next train_step replays it

    def train_step(self) -> None:
        """Run one optimizer step on the next batch (asynchronously)."""
        self._write_batch(self.steps_done)
        if self._graph is not None:
            self._graph.replay()
        else:
            self._body()
        self.steps_done += 1

    def log_row(self) -> dict[str, float]:
        row = {"step": self.steps_done, "loss": float(self.loss)}
        row.update({k: float(v) for k, v in self.components.items()})
        row["grad_norm"] = float(self.opt.state[3])
        return row

    def release(self) -> None:
        self._graph = None
        from .deferred_grad import restore_linears

        restore_linears(self.stash)
        self.stash = None
        if self.group is not None:
            torch.cuda.synchronize(self.device)
            self.group.close()

    # ------------------------------------------------------------ checkpoint
    def save(self, path: Path | str, *, training_args: dict | None = None) -> None:
        """Adapter checkpoint (reference format) plus this rank's optimizer shard."""
        ckpt = build_adapter_checkpoint(self.model, completed_steps=self.steps_done,
                                        training_args=training_args or self.cfg.to_dict(),
                                        extra={"optimizer": self.opt.state_dict(), "world": self.world,
                                               "rank": self.rank})
        path = Path(path)
        tmp = path.with_suffix(path.suffix + ".tmp")
        torch.save(ckpt, tmp)
        tmp.replace(path)

    def resume(self, path: Path | str, *, restore_optimizer: bool = True) -> dict[str, Any]:
        ckpt = load_adapter_checkpoint(self.model, path)
        self.steps_done = int(ckpt.get("completed_steps", 0))
        opt = ckpt.get("optimizer")
        if restore_optimizer and opt is not None and ckpt.get("world") == self.world:
            self.opt.load_state_dict(opt)
            if self.world > 1 and not self.nccl:  # flags restart at epoch 0; the bias correction continues
                self.opt.hyper[6].fill_(float(opt["state"][0]))
        return ckpt


# --------------------------------------------------------------- evaluation
@torch.no_grad()
def evaluate_drafter(model: SparseKVEagleDrafter, bank: DeviceTeacherBank, rows: Sequence[int], rope_cos, rope_sin,
                     *, memory_mode: str = "exact", draft_tokens: int = 4, teacher_forced_tokens: int = 8,
                     batch: int = 64) -> dict[str, Any]:
    """Teacher-forced top-1 and accepted prefix of ``draft_tokens``-token greedy drafts."""
    if memory_mode not in {"exact", "zero", "shuffled", "disabled"}:
        raise ValueError("unsupported EAGLE memory ablation")
    dev = bank.input_ids.device
    groups = bank.groups or list(range(bank.size))
    accepted, correct, covered_correct, covered, total = [], 0, 0, 0, 0
    cos_t = rope_cos.to(dev, torch.bfloat16)
    sin_t = rope_sin.to(dev, torch.bfloat16)
    for i in range(0, len(rows), batch):
        chunk = list(rows[i:i + batch])
        idx = torch.tensor(chunk, device=dev)
        mem_rows = idx if memory_mode != "shuffled" else torch.tensor(
            [pick_mismatched(groups, r) for r in chunk], device=dev)
        mem = MemoryBatch(bank.mem_k, bank.mem_v, bank.idx, bank.n_vis, mem_rows.to(torch.int32),
                          zero=memory_mode == "zero")
        use_mem = memory_mode != "disabled"
        t = min(teacher_forced_tokens, bank.horizon)
        ids = bank.input_ids.index_select(0, idx)
        labels = bank.labels.index_select(0, idx)
        pos = bank.prompt_tokens.index_select(0, idx)[:, None] + torch.arange(max(t, draft_tokens), device=dev)
        cos, sin = cos_t[pos], sin_t[pos]
        seeds = bank.seed_hidden.index_select(0, idx).to(model.fc.weight.dtype)
        stage = bank.stage(idx)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=dev.type == "cuda"):
            feats = model.recurrent_forward(ids[:, :t], seeds, mem, None, cos[:, :t], sin[:, :t], stage,
                                            use_memory=use_mem)
            pred = model.target_ids(model.lm_head(feats).argmax(-1))
            ok = model.draft_ids(labels[:, :t]) >= 0
            hit = pred == labels[:, :t]
            correct += int(hit.sum())
            covered_correct += int((hit & ok).sum())
            covered += int(ok.sum())
            total += hit.numel()
            n = min(draft_tokens, bank.horizon)
            prop = model.propose(ids[:, :1], seeds, mem, None, cos[:, :n], sin[:, :n], stage, n_tokens=n,
                                 use_memory=use_mem)
        for p, lab in zip(prop.tolist(), labels[:, :n].tolist()):
            accepted.append(accepted_prefix_length(p, lab))
    return {
        "memory_mode": memory_mode,
        "samples": len(rows),
        "draft_tokens": draft_tokens,
        "teacher_forced_top1": correct / max(total, 1),
        "covered_teacher_forced_top1": covered_correct / max(covered, 1),
        "label_coverage": covered / max(total, 1),
        "mean_accepted_prefix": sum(accepted) / max(len(accepted), 1),
        "full_accept_rate": sum(a == min(draft_tokens, bank.horizon) for a in accepted) / max(len(accepted), 1),
    }


def random_eagle_drafter(cfg: SparseKVEagleConfig, *, seed: int = 0, std: float = 0.02) -> SparseKVEagleDrafter:
    """A random-init EAGLE trunk (no pretrained checkpoint available offline) with an
    identity draft vocabulary map over the first ``draft_vocab_size`` target ids."""
    torch.manual_seed(seed)
    model = SparseKVEagleDrafter(cfg)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.ndim == 2 and not name.startswith(("memory_gate", "memory_delta", "stage_layer_bias")):
                p.normal_(0.0, std)
        model.d2t.zero_()
        model._rebuild_vocab_maps()
    return model


def write_json(path: Path | str, payload: dict) -> None:
    Path(path).write_text(json.dumps(payload, indent=2, sort_keys=True) + "\n", encoding="utf-8")


def log2_prompt_feature(prompt_tokens: int) -> float:
    return math.log2(prompt_tokens + 1) / 17.0
