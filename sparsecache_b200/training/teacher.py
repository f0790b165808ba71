"""Drafter teacher data: reference formats, memory views, and a device bank.

Reference-format side (parity with experiments/train_sparse_kv_drafter.py):
  * ``load_teacher_dataset`` reads ``sparsecache.sparse-kv-draft-teacher.v1..v5``
    manifests, checks every file's sha256, merges v4/v5 traces with their v3
    static-KV base manifest and validates the exact field set per version
    (:175-291);
  * ``select_memory`` = page selection + gather of the visible token rows
    (:294-316); ``sample_inputs`` / ``training_window_inputs`` give the
    initial or post-verification-boundary window (:319-379).

B200 side:
  * ``DeviceTeacherBank`` keeps a whole training set resident in HBM: each
    request's memory is cut at build time to its visible view (by default 64
    sink + 512 recent + top-scored 64-token chunks, 2048 tokens in all) and
    stored token-major [S, L, V, H, 128] bf16, so a training step reads K/V
    rows in place through ``MemoryBatch`` instead of gathering on the CPU and
    copying per step as the reference does;
  * ``extract_teacher`` produces the teacher fields with this package's
    engine on the GPU: one prefill of the prompt (memory layers' K/V, the
    seed layers' last hidden states, the K11 page scores of the last
    prompt token's queries), a greedy continuation decoded with the CUDA
    graph decode path, and one prefill of the continuation over the cached
    prompt for the teacher logits (top-k) and final hidden states.
"""
from __future__ import annotations

import hashlib
import json
import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Sequence

import torch
import torch.nn.functional as F

from .. import ops

from ..models.sparse_kv_draft import select_visible_token_indices, sink_recent_topk_indices

TEACHER_FORMATS = tuple(f"sparsecache.sparse-kv-draft-teacher.v{i}" for i in range(1, 6))
_BASE_FIELDS = {"memory_keys", "memory_values", "seed_hidden", "input_ids", "labels", "teacher_topk_ids",
                "teacher_topk_logprobs", "query_cos", "query_sin", "prompt_ids"}
_STATIC_FIELDS = {"memory_keys", "memory_values", "seed_hidden", "priority_page_scores", "prompt_ids"}
_INITIAL_FIELDS = {"input_ids", "labels", "teacher_topk_ids", "teacher_topk_logprobs", "teacher_hidden",
                   "query_cos", "query_sin"}


def required_fields(version: int) -> set[str]:
    req = set(_BASE_FIELDS)
    if version == 2:
        req.add("teacher_hidden")
    if version in (3, 4):
        req |= {"teacher_hidden", "priority_page_scores"}
    if version == 5:
        req |= {"teacher_hidden", "priority_page_scores", "continuation_seed_hidden"}
    return req


def sha256_file(path: str | Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


@dataclass
class TeacherSample:
    request_index: int
    prompt_tokens: int
    tensors: dict[str, torch.Tensor]
    source_group: str | None = None

    @property
    def horizon(self) -> int:
        return int(self.tensors["labels"].numel())


def load_teacher_dataset(manifest_path: Path | str, requested_indices: set[int] | None = None):
    """Load (and hash-check) a reference-format teacher manifest -> (manifest, {index: sample})."""
    from safetensors.torch import load_file

    manifest_path = Path(manifest_path)
    manifest = json.loads(manifest_path.read_text(encoding="utf-8"))
    fmt = manifest.get("format")
    if fmt not in TEACHER_FORMATS:
        raise ValueError("unsupported teacher-data format")
    version = int(fmt.rsplit(".v", 1)[1])
    root = manifest_path.parent
    base_rows: dict[int, dict] = {}
    base_root = root
    if version >= 4:
        base_path = Path(manifest["base_manifest"])
        base = json.loads(base_path.read_text(encoding="utf-8"))
        if base.get("format") != TEACHER_FORMATS[2]:
            raise ValueError("v4 teacher data requires a v3 static-KV manifest")
        if base.get("target_fingerprint") != manifest.get("target_fingerprint"):
            raise ValueError("v4 trace and static KV target fingerprints differ")
        base_root = base_path.parent
        base_rows = {int(r["request_index"]): r for r in base["samples"]}
    samples: dict[int, TeacherSample] = {}
    for row in manifest.get("samples", []):
        index = int(row["request_index"])
        if requested_indices is not None and index not in requested_indices:
            continue
        if index in samples:
            raise ValueError(f"duplicate teacher request {index}")
        path = root / row["file"]
        if sha256_file(path) != row.get("file_sha256"):
            raise ValueError(f"teacher request {index} hash differs")
        tensors = dict(load_file(str(path), device="cpu"))
        base_tensors = None
        if version >= 4:
            brow = base_rows.get(index)
            if brow is None:
                raise ValueError(f"teacher request {index} has no static KV")
            bpath = base_root / brow["file"]
            if sha256_file(bpath) != brow.get("file_sha256"):
                raise ValueError(f"static KV request {index} hash differs")
            base_tensors = load_file(str(bpath), device="cpu")
            tensors.update({k: base_tensors[k] for k in _STATIC_FIELDS})
        if set(tensors) != required_fields(version):
            raise ValueError(f"teacher request {index} has invalid fields")
        if version == 5:
            tensors.update({f"initial_{k}": base_tensors[k] for k in _INITIAL_FIELDS})
        prompt_tokens = int(tensors["prompt_ids"].numel())
        if prompt_tokens != int(row["prompt_tokens"]):
            raise ValueError(f"teacher request {index} length differs")
        samples[index] = TeacherSample(index, prompt_tokens, tensors, row.get("source_dataset"))
    if not samples:
        raise ValueError("teacher manifest contains no samples")
    return manifest, samples


def select_memory(sample: TeacherSample, *, page_size: int, requested_fraction: float, seed: int, device,
                  selection_mode: str = "random"):
    """(keys, values, actual_fraction, visible_tokens) of one sparse page view."""
    idx = select_visible_token_indices(
        sample.prompt_tokens, page_size=page_size, visible_fraction=requested_fraction, seed=seed,
        protected_prefix_pages=1, protected_suffix_pages=1, mode=selection_mode,
        page_scores=sample.tensors.get("priority_page_scores"))
    keys = sample.tensors["memory_keys"].index_select(2, idx).to(device)
    values = sample.tensors["memory_values"].index_select(2, idx).to(device)
    n = int(idx.numel())
    return keys, values, n / sample.prompt_tokens, n


def sample_inputs(sample: TeacherSample, device):
    """(input_ids [1,t], seed_hidden [1,S,H], cos, sin, labels, topk ids, topk logprobs) of the first window."""
    t = sample.tensors
    p = "initial_" if "initial_input_ids" in t else ""
    return (t[f"{p}input_ids"].to(device).unsqueeze(0), t["seed_hidden"].to(device).unsqueeze(0),
            t[f"{p}query_cos"].to(device), t[f"{p}query_sin"].to(device), t[f"{p}labels"].to(device),
            t[f"{p}teacher_topk_ids"].to(device), t[f"{p}teacher_topk_logprobs"].to(device))


def training_window_inputs(sample: TeacherSample, device, *, offset: int, window_tokens: int):
    """A window of the continuation: offset 0 starts at the prompt seed, later
    offsets start from the verifier's boundary hidden states (v5 data)."""
    if window_tokens <= 0 or not 0 <= offset < sample.horizon:
        raise ValueError("invalid teacher-window bounds")
    if offset == 0:
        full = sample_inputs(sample, device)
        stop = min(full[0].shape[1], window_tokens)
        return (full[0][:, :stop], full[1], full[2][:stop], full[3][:stop], full[4][:stop], full[5][:stop],
                full[6][:stop])
    t = sample.tensors
    cont = t.get("continuation_seed_hidden")
    if cont is None:
        raise ValueError("windowed training requires v5 boundary hidden states")
    if tuple(cont.shape) != (sample.horizon, *t["seed_hidden"].shape):
        raise ValueError("continuation boundary hidden states have invalid shape")
    stop = min(sample.horizon, offset + window_tokens)
    return (t["input_ids"][offset:stop].to(device).unsqueeze(0), cont[offset - 1].to(device).unsqueeze(0),
            t["query_cos"][offset:stop].to(device), t["query_sin"][offset:stop].to(device),
            t["labels"][offset:stop].to(device), t["teacher_topk_ids"][offset:stop].to(device),
            t["teacher_topk_logprobs"][offset:stop].to(device))


def pick_mismatched(groups: Sequence[Any], index: int) -> int:
    """Index of the next sample from another source group (else simply the next one)."""
    n = len(groups)
    for off in range(1, n):
        j = (index + off) % n
        if groups[j] != groups[index]:
            return j
    return (index + 1) % n


# ------------------------------------------------------------------ device bank
@dataclass
class DeviceTeacherBank:
    """A training set resident on one GPU (see module docstring)."""

    mem_k: torch.Tensor            # [S, L, V, H, D] bf16
    mem_v: torch.Tensor
    idx: torch.Tensor              # [S, V] int32 visible rows (into mem_k's V axis)
    n_vis: torch.Tensor            # [S] int32
    seed_hidden: torch.Tensor      # [S, n_seed, Ht] bf16
    input_ids: torch.Tensor        # [S, t] int64
    labels: torch.Tensor           # [S, t] int64
    topk_ids: torch.Tensor         # [S, t, k] int64
    topk_logprobs: torch.Tensor    # [S, t, k] fp32
    prompt_tokens: torch.Tensor    # [S] int64 (first continuation position)
    visible_fraction: torch.Tensor  # [S] fp32
    teacher_hidden: torch.Tensor | None = None  # [S, t, H] bf16
    groups: list = field(default_factory=list)

    @property
    def size(self) -> int:
        return self.input_ids.shape[0]

    @property
    def horizon(self) -> int:
        return self.input_ids.shape[1]

    def stage(self, rows: torch.Tensor) -> torch.Tensor:
        """[B, 2] stage features (visible fraction, log2(P+1)/17) of bank rows."""
        frac = self.visible_fraction.index_select(0, rows)
        p = self.prompt_tokens.index_select(0, rows).float()
        return torch.stack((frac, torch.log2(p + 1.0) / 17.0), dim=-1)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.mem_k, self.mem_v, self.seed_hidden, self.input_ids,
                                                          self.labels, self.topk_ids, self.topk_logprobs))


def _stack_views(views: list[tuple[torch.Tensor, torch.Tensor]], device) -> tuple[torch.Tensor, ...]:
    """Pad per-sample [L, H, n, D] views to [S, L, V, H, D] token-major + idx/n_vis."""
    V = max(k.shape[2] for k, _ in views)
    S = len(views)
    L, H, _, D = views[0][0].shape
    mk = torch.zeros(S, L, V, H, D, dtype=torch.bfloat16, device=device)
    mv = torch.zeros_like(mk)
    n_vis = torch.empty(S, dtype=torch.int32)
    for s, (k, v) in enumerate(views):
        n = k.shape[2]
        mk[s, :, :n] = k.to(device=device, dtype=torch.bfloat16).permute(0, 2, 1, 3)
        mv[s, :, :n] = v.to(device=device, dtype=torch.bfloat16).permute(0, 2, 1, 3)
        n_vis[s] = n
    idx = torch.arange(V, dtype=torch.int32).repeat(S, 1)
    return mk, mv, idx.to(device), n_vis.to(device)


def bank_from_samples(samples: Sequence[TeacherSample], device, *, view: str = "sink_recent_topk",
                      page_size: int = 64, fraction: float = 0.1, seed: int = 0, sink: int = 64,
                      recent: int = 512, budget: int = 2048) -> DeviceTeacherBank:
    """Cut each sample's memory to its view and move the set to ``device``."""
    views, fracs = [], []
    for i, s in enumerate(samples):
        if view == "sink_recent_topk":
            scores = s.tensors.get("priority_page_scores")
            if scores is not None and page_size != 64:
                raise ValueError("chunk scores are per 64-token page")
            idx = sink_recent_topk_indices(s.prompt_tokens, scores, sink=sink, recent=recent, chunk=64,
                                           budget=budget)
        else:
            idx = select_visible_token_indices(s.prompt_tokens, page_size=page_size, visible_fraction=fraction,
                                               seed=seed + s.request_index * 1009, mode=view,
                                               page_scores=s.tensors.get("priority_page_scores"))
        views.append((s.tensors["memory_keys"].index_select(2, idx), s.tensors["memory_values"].index_select(2, idx)))
        fracs.append(idx.numel() / s.prompt_tokens)
    mk, mv, idx, n_vis = _stack_views(views, device)
    horizon = min(s.horizon for s in samples)

    def stack(name, dtype=None):
        return torch.stack([s.tensors[name][:horizon] for s in samples]).to(device=device, dtype=dtype)

    th = None
    if all("teacher_hidden" in s.tensors for s in samples):
        th = stack("teacher_hidden", torch.bfloat16)
    return DeviceTeacherBank(
        mem_k=mk, mem_v=mv, idx=idx, n_vis=n_vis,
        seed_hidden=torch.stack([s.tensors["seed_hidden"] for s in samples]).to(device=device, dtype=torch.bfloat16),
        input_ids=stack("input_ids", torch.int64), labels=stack("labels", torch.int64),
        topk_ids=stack("teacher_topk_ids", torch.int64), topk_logprobs=stack("teacher_topk_logprobs", torch.float32),
        prompt_tokens=torch.tensor([s.prompt_tokens for s in samples], dtype=torch.int64, device=device),
        visible_fraction=torch.tensor(fracs, dtype=torch.float32, device=device),
        teacher_hidden=th, groups=[s.source_group for s in samples])


def synthetic_bank(*, n_samples: int, horizon: int, n_layers: int, n_heads: int, n_seed: int, target_hidden: int,
                   hidden: int, vocab: int, visible: int, prompt_tokens: int, topk: int, device,
                   seed: int = 0, head_dim: int = 128) -> DeviceTeacherBank:
    """Random teacher data of the given geometry, generated on ``device`` (for
    tests and for timing the trainer without a teacher run)."""
    g = torch.Generator(device=device).manual_seed(seed)
    D = head_dim

    def rn(*shape, dtype=torch.bfloat16, scale=1.0):
        return (torch.randn(*shape, generator=g, device=device) * scale).to(dtype)

    ids = torch.randint(0, vocab, (n_samples, horizon + 1), generator=g, device=device)
    topk_ids = torch.randint(0, vocab, (n_samples, horizon, topk), generator=g, device=device)
    topk_ids[..., 0] = ids[:, 1:]
    lp = torch.randn(n_samples, horizon, topk, generator=g, device=device).sort(-1, descending=True).values
    return DeviceTeacherBank(
        mem_k=rn(n_samples, n_layers, visible, n_heads, D), mem_v=rn(n_samples, n_layers, visible, n_heads, D),
        idx=torch.arange(visible, dtype=torch.int32, device=device).repeat(n_samples, 1),
        n_vis=torch.full((n_samples,), visible, dtype=torch.int32, device=device),
        seed_hidden=rn(n_samples, n_seed, target_hidden),
        input_ids=ids[:, :-1].contiguous(), labels=ids[:, 1:].contiguous(), topk_ids=topk_ids,
        topk_logprobs=lp.log_softmax(-1),
        prompt_tokens=torch.full((n_samples,), prompt_tokens, dtype=torch.int64, device=device),
        visible_fraction=torch.full((n_samples,), visible / prompt_tokens, dtype=torch.float32, device=device),
        teacher_hidden=rn(n_samples, horizon, hidden), groups=[i % 4 for i in range(n_samples)])


# -------------------------------------------------------------- GPU extraction
def page_scores_from_queries(q: torch.Tensor, keys: torch.Tensor, n_tokens: int, page_size: int) -> torch.Tensor:
    """K11: mean over heads of softmax(q.K^T * d^-0.5) of one query row, summed per page.

    ``q`` [Hq, D] (RoPE applied), ``keys`` [Hkv, T, D]; GQA groups of query
    heads share a key head.  Returns [ceil(T / page_size)] fp32.
    """
    hq, d = q.shape
    hkv = keys.shape[0]
    k = keys[:, :n_tokens].float()
    qg = q.float().view(hkv, hq // hkv, d)
    probs = torch.einsum("gqd,gkd->gqk", qg, k).mul(d ** -0.5).softmax(-1)
    tok = probs.mean(dim=(0, 1))
    pages = -(-n_tokens // page_size)
    tok = F.pad(tok, (0, pages * page_size - n_tokens))
    return tok.view(pages, page_size).sum(-1)


@torch.no_grad()
def extract_teacher(engine, prompts: Sequence[torch.Tensor], *, kv_layers: Sequence[int],
                    seed_layers: Sequence[int], continuation_tokens: int, teacher_topk: int = 64,
                    page_size: int = 64, keep_full_memory: bool = False, view_budget: int = 2048,
                    sink: int = 64, recent: int = 512, slot=None) -> list[TeacherSample]:
    """Teacher samples of ``prompts`` (int32 token tensors) from the engine's target model.

    Fields follow the v3 teacher format (memory keys/values [L, H, T, D] of
    ``kv_layers``, ``seed_hidden`` [len(seed_layers), d], greedy
    ``input_ids``/``labels``, top-k ids/log-probs, the final normalised
    ``teacher_hidden``, ``priority_page_scores``, query cos/sin of the
    continuation positions, ``prompt_ids``).  Unless ``keep_full_memory``, the
    memory is cut at once to the sink/recent/top-chunk view (then the view's
    token indices are stored as ``memory_token_index``), which keeps a 16k
    context's teacher record at the size of 2048 tokens.
    """
    from ..rope import rope_cos_sin, apply_rope

    cfg = engine.cfg
    dev = engine.device
    w = engine.w
    samples = []
    for i, prompt in enumerate(prompts):
        prompt = prompt.to(device=dev, dtype=torch.int32)
        T = prompt.numel()
        cap = T + continuation_tokens + 64
        s = slot if slot is not None and slot.capacity >= cap else engine.new_slot(cap)
        captured: dict[int, torch.Tensor] = {}

        def hook(layer: int, h: torch.Tensor) -> None:
            if layer - 1 in seed_layers:
                captured[layer - 1] = h[T - 1].clone()
            if layer in kv_layers:
                captured[("q", layer)] = h[T - 1].clone()

        h = engine.prefill(prompt, s, layer_hook=hook)
        if cfg.n_layers - 1 in seed_layers:
            captured[cfg.n_layers - 1] = h[T - 1].clone()
        seed_hidden = torch.stack([captured[l] for l in seed_layers])
        # K11 page scores: the last prompt token's queries of every memory layer
        cos, sin = rope_cos_sin(cfg, torch.tensor([T - 1]), device=dev)
        queries = []
        for l in kv_layers:
            x = captured[("q", l)].float()
            x = x * torch.rsqrt(x.square().mean() + cfg.rms_eps)
            x = (x.to(torch.bfloat16) * w.layers[l].ln1).float()
            q = (w.layers[l].w_qkv[: cfg.q_size].float() @ x).view(cfg.n_heads, cfg.head_dim)
            queries.append(apply_rope(q.unsqueeze(1), cos, sin, sequence_dim=1).squeeze(1))
        # K11 on the GPU: layer-mean token scores, then per-page sums
        tok = ops.ext().page_token_scores(torch.stack(queries).unsqueeze(1).contiguous(),
                                          [s.k(l) for l in kv_layers], T, cfg.head_dim ** -0.5)
        pages = -(-T // page_size)
        scores = F.pad(tok, (0, pages * page_size - T)).view(pages, page_size).sum(-1)
        # greedy continuation (CUDA-graph decode), then one prefill of it for the teacher logits
        engine.first_token(h[T - 1:T], position=T, max_new=continuation_tokens)
        engine.decode(s, continuation_tokens - 1, max_new=continuation_tokens)
        input_ids = engine.generated_tokens(continuation_tokens).clone().to(torch.int32)
        boundary: dict[int, torch.Tensor] = {}

        def cont_hook(layer: int, hh: torch.Tensor) -> None:
            if layer - 1 in seed_layers:
                boundary[layer - 1] = hh.clone()

        hc = engine.prefill(input_ids, s, start=T, layer_hook=cont_hook)
        if cfg.n_layers - 1 in seed_layers:
            boundary[cfg.n_layers - 1] = hc.clone()
        # seed-layer hidden states after every continuation token: the
        # post-verification boundary features of windowed training (v5)
        cont_seed = torch.stack([boundary[l] for l in seed_layers], dim=1)  # [t, seeds, d]
        x = hc.float()
        normed = (x * torch.rsqrt(x.square().mean(-1, keepdim=True) + cfg.rms_eps)).to(torch.bfloat16) * w.norm
        logits = (normed @ w.lm_head.t()).float()
        lp = logits.log_softmax(-1)
        top_lp, top_ids = lp.topk(teacher_topk, dim=-1)
        labels = logits.argmax(-1)
        mk = torch.stack([s.k(l)[:, :T] for l in kv_layers])  # [L, H, T, D]
        mv = torch.stack([s.v(l)[:, :T] for l in kv_layers])
        tensors = {}
        if not keep_full_memory:
            view = sink_recent_topk_indices(T, scores.cpu(), sink=sink, recent=recent, chunk=page_size,
                                            budget=view_budget).to(dev)
            mk, mv = mk.index_select(2, view), mv.index_select(2, view)
            tensors["memory_token_index"] = view.cpu().to(torch.int32)
        positions = torch.arange(T, T + input_ids.numel())
        qc, qs = rope_cos_sin(cfg, positions, dtype=torch.bfloat16)
        tensors.update({
            "memory_keys": mk.cpu(), "memory_values": mv.cpu(), "seed_hidden": seed_hidden.cpu(),
            "input_ids": input_ids.long().cpu(), "labels": labels.long().cpu(),
            "teacher_topk_ids": top_ids.long().cpu(), "teacher_topk_logprobs": top_lp.cpu(),
            "teacher_hidden": normed.cpu(), "priority_page_scores": scores.float().cpu(),
            "query_cos": qc, "query_sin": qs, "prompt_ids": prompt.cpu(),
            "continuation_seed_hidden": cont_seed.cpu()})
        samples.append(TeacherSample(i, T, tensors, None))
    return samples


def _oracle_layers(model, ids: torch.Tensor, positions: torch.Tensor, past=None):
    """Oracle layer loop -> (hidden entering every layer + final hidden, [T, d] each; new cache)."""
    hidden = model.embed_tokens(ids.to(model.device).view(1, -1))
    positions = positions.to(model.device)
    cos, sin = model.rope(positions)
    key_pos = positions if past is None else torch.cat(
        (torch.arange(past[0][0].shape[2], device=model.device), positions))
    entering, cache = [], []
    for index, layer in enumerate(model.layers):
        entering.append(hidden[0])
        q, k, v = model.project_qkv(layer, layer.input_layernorm(hidden), cos, sin)
        if past is not None:
            k = torch.cat((past[index][0], k), dim=2)
            v = torch.cat((past[index][1], v), dim=2)
        attended = model.attention(q, k, v, query_positions=positions, key_positions=key_pos)
        hidden = model.block_rest(layer, hidden, attended)
        cache.append((k, v))
    entering.append(hidden[0])
    return entering, tuple(cache)


@torch.no_grad()
def extract_teacher_oracle(model, prompts: Sequence[torch.Tensor], *, kv_layers: Sequence[int],
                           seed_layers: Sequence[int], continuation_tokens: int, teacher_topk: int = 64,
                           page_size: int = 64,
                           continuation_ids: Sequence[torch.Tensor] | None = None) -> list[TeacherSample]:
    """``extract_teacher`` restated on the plain-PyTorch oracle model (``models.llama.LlamaOracle``).

    Same fields and storage dtypes as the engine path with the full prompt
    memory (reference: experiments/extract_sparse_kv_teacher.py:97-323 for
    the v3 fields, experiments/extend_sparse_kv_teacher.py:28-136 for
    ``continuation_seed_hidden``): the numerics oracle of the GPU extractor
    and the CPU path of the extraction command line.  ``continuation_ids``
    (one token tensor per prompt) replaces the greedy continuation, so the
    teacher fields can be compared along another extractor's tokens.
    """
    from ..rope import apply_rope

    cfg = model.config
    bf = torch.bfloat16
    samples = []
    for i, prompt in enumerate(prompts):
        ids = prompt.to(torch.long).cpu()
        T = ids.numel()
        entering, cache = _oracle_layers(model, ids, torch.arange(T))
        seed_hidden = torch.stack([entering[s + 1][T - 1] for s in seed_layers])
        cos, sin = model.rope(torch.tensor([T - 1]))
        page_probs = []
        for l in kv_layers:
            layer = model.layers[l]
            q = layer.q_proj(layer.input_layernorm(entering[l][T - 1:T])).view(cfg.n_heads, 1, cfg.head_dim)
            q = apply_rope(q, cos, sin, sequence_dim=1).squeeze(1)
            page_probs.append(page_scores_from_queries(q, cache[l][0][0], T, page_size))
        scores = torch.stack(page_probs).mean(0)
        # greedy continuation token by token, then one pass over it for the teacher fields
        if continuation_ids is not None:
            input_ids = continuation_ids[i].to(torch.long).cpu()
        else:
            tokens = [int(model.logits(entering[-1][T - 1:T]).float().argmax())]
            past = cache
            for step in range(continuation_tokens - 1):
                hid, past = model.forward_tokens(torch.tensor([tokens[-1]]), torch.tensor([T + step]), past=past)
                tokens.append(int(model.logits(hid[:, -1]).float().argmax()))
            input_ids = torch.tensor(tokens, dtype=torch.long)
        n = input_ids.numel()
        cont, _ = _oracle_layers(model, input_ids, torch.arange(T, T + n), past=cache)
        normed = model.norm(cont[-1])
        logits = model.lm_head(normed).float()
        lp = logits.log_softmax(-1)
        top_lp, top_ids = lp.topk(teacher_topk, dim=-1)
        qc, qs = model.rope(torch.arange(T, T + n))
        tensors = {
            "memory_keys": torch.stack([cache[l][0][0] for l in kv_layers]).to(bf),
            "memory_values": torch.stack([cache[l][1][0] for l in kv_layers]).to(bf),
            "seed_hidden": seed_hidden.to(bf), "input_ids": input_ids, "labels": logits.argmax(-1),
            "teacher_topk_ids": top_ids.long(), "teacher_topk_logprobs": top_lp.float(),
            "teacher_hidden": normed.to(bf), "priority_page_scores": scores.float(),
            "query_cos": qc.to(bf), "query_sin": qs.to(bf), "prompt_ids": ids.to(torch.int32),
            "continuation_seed_hidden": torch.stack([cont[s + 1] for s in seed_layers], dim=1).to(bf)}
        samples.append(TeacherSample(i, T, tensors, None))
    return samples


_TRACE_FIELDS = ("input_ids", "labels", "teacher_topk_ids", "teacher_topk_logprobs", "teacher_hidden",
                 "query_cos", "query_sin", "continuation_seed_hidden")


def truncate_at_eos(tensors: dict[str, torch.Tensor], eos: set[int]) -> dict[str, torch.Tensor]:
    """Cut the continuation after the first label in ``eos`` (kept), as a greedy teacher that stops there."""
    labels = tensors["labels"].tolist()
    stop = next((j + 1 for j, t in enumerate(labels) if t in eos), len(labels))
    if stop == len(labels):
        return tensors
    return {k: (v[:stop] if k in _TRACE_FIELDS else v) for k, v in tensors.items()}


def prompt_sha256(prompt_ids: Sequence[int]) -> str:
    """sha256 of the compact JSON list of prompt ids (the reference's per-sample prompt hash)."""
    return hashlib.sha256(json.dumps([int(t) for t in prompt_ids], separators=(",", ":")).encode()).hexdigest()


def bank_from_extracted(samples: Sequence[TeacherSample], device) -> DeviceTeacherBank:
    """Bank of ``extract_teacher`` output whose memory is already cut to its view."""
    views = [(s.tensors["memory_keys"], s.tensors["memory_values"]) for s in samples]
    mk, mv, idx, n_vis = _stack_views(views, device)
    horizon = min(s.horizon for s in samples)

    def stack(name, dtype):
        return torch.stack([s.tensors[name][:horizon] for s in samples]).to(device=device, dtype=dtype)

    return DeviceTeacherBank(
        mem_k=mk, mem_v=mv, idx=idx, n_vis=n_vis,
        seed_hidden=torch.stack([s.tensors["seed_hidden"] for s in samples]).to(device=device, dtype=torch.bfloat16),
        input_ids=stack("input_ids", torch.int64), labels=stack("labels", torch.int64),
        topk_ids=stack("teacher_topk_ids", torch.int64), topk_logprobs=stack("teacher_topk_logprobs", torch.float32),
        prompt_tokens=torch.tensor([s.prompt_tokens for s in samples], dtype=torch.int64, device=device),
        visible_fraction=torch.tensor([s.tensors["memory_keys"].shape[2] / s.prompt_tokens for s in samples],
                                      dtype=torch.float32, device=device),
        teacher_hidden=stack("teacher_hidden", torch.bfloat16), groups=[s.source_group for s in samples])


def visible_fraction_of(n_visible: int, prompt_tokens: int) -> float:
    return min(1.0, n_visible / max(prompt_tokens, 1))


def chunk_count(prompt_tokens: int, chunk: int = 64) -> int:
    return math.ceil(prompt_tokens / chunk)


def _atomic_save(tensors: dict[str, torch.Tensor], path: Path) -> None:
    from safetensors.torch import save_file

    tmp = path.with_suffix(path.suffix + ".tmp")
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(tmp))
    tmp.replace(path)


def write_teacher_dataset(samples: Sequence[TeacherSample], out_dir: Path, *, target_fingerprint: str,
                          kv_layers: Sequence[int], seed_layers: Sequence[int], head_dim: int, kv_heads: int,
                          target_hidden_size: int, vocab_size: int, priority_page_size: int = 64,
                          target_model: str = "random-init", with_boundaries: bool = False) -> Path:
    """Write samples in the reference's teacher format; returns the manifest path.

    Static K/V and traces go to a v3 manifest; with ``with_boundaries`` a v5
    manifest is written next to it that chains to the v3 one (traces plus
    ``continuation_seed_hidden``), as the reference's extender does.  Memory
    must be the full prompt's K/V (not a cut view).
    """
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    v3 = required_fields(3)
    rows, rows5 = [], []
    for s in samples:
        if "memory_token_index" in s.tensors:
            raise ValueError("the reference format stores the full prompt memory (extract with keep_full_memory)")
        f = out_dir / f"sample_{s.request_index:05d}.safetensors"
        _atomic_save({k: s.tensors[k] for k in v3}, f)
        rows.append({"request_index": s.request_index, "file": f.name, "prompt_tokens": s.prompt_tokens,
                     "draft_training_tokens": s.horizon, "file_sha256": sha256_file(f),
                     "source_dataset": s.source_group})
        if with_boundaries:
            f5 = out_dir / f"trace_{s.request_index:05d}.safetensors"
            trace = {k: s.tensors[k] for k in required_fields(5) - _STATIC_FIELDS}
            _atomic_save(trace, f5)
            rows5.append({**rows[-1], "file": f5.name, "file_sha256": sha256_file(f5)})
    common = {"target_model": target_model, "target_fingerprint": target_fingerprint, "kv_layers": list(kv_layers),
              "seed_layers": list(seed_layers), "head_dim": head_dim, "kv_heads": kv_heads,
              "target_hidden_size": target_hidden_size, "vocab_size": vocab_size,
              "priority_page_size": priority_page_size}
    m3 = out_dir / "manifest.json"
    m3.write_text(json.dumps({"schema_version": 3, "format": TEACHER_FORMATS[2], **common, "samples": rows},
                             indent=2, sort_keys=True) + "\n")
    if not with_boundaries:
        return m3
    m5 = out_dir / "manifest_v5.json"
    m5.write_text(json.dumps({"schema_version": 5, "format": TEACHER_FORMATS[4], "base_manifest": str(m3.resolve()),
                              **common, "samples": rows5}, indent=2, sort_keys=True) + "\n")
    return m5
