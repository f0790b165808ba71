"""EAGLE-3 language prior conditioned on exact sparse verifier KV.

Behavioural parity with the reference's src/sparsecache/sparse_kv_eagle.py:
``SparseKVEagleConfig`` (:26-66), ``EagleSelfAttention`` (:69-121),
``EagleMLP`` (:124-138), ``EagleDraftLayer`` (:141-170) and
``SparseKVEagleDrafter`` (:173-410): the frozen EAGLE trunk (fc over the seed
layers, one recurrent mid-layer whose attention input is
``[input_norm(embedding) || hidden_norm(hidden)]``, final norm, compressed
LM head) plus a trainable adapter that issues queries into selected target
KV layers and adds ``sigmoid(adapter_scale) * delta`` (scalar fusion) or a
gated correction (gated-delta fusion) to the recurrent hidden state.
Parameter and buffer names match the reference so EAGLE checkpoints and
adapter checkpoints load unchanged.

The trunk is recurrent: the hidden state of position p is the mid-layer
output of position p-1.  ``forward`` keeps the reference's batch-1 API;
``recurrent_forward`` is the batched form (any number of rows, each with its
own memory view, stage features and RoPE positions) that the trainer and the
evaluator drive, and that ``forward`` itself calls.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops.linear import recurrent_attention
from ..rope import apply_rope
from .sparse_kv_draft import RMSNorm, SparseKVDraftConfig, SparseTargetKVAttention, stage_features


# how the adapter's memory read joins the recurrent hidden state (see
# SparseKVEagleDrafter.fuse): "scalar" adds sigmoid(adapter_scale) * delta;
# "gated_delta" adds a gated, linearly mapped correction toward delta
FUSION_MODES = frozenset({"scalar", "gated_delta"})


@dataclass(frozen=True)
class SparseKVEagleConfig:
    target_hidden_size: int = 4096
    hidden_size: int = 4096
    intermediate_size: int = 14336
    head_dim: int = 128
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    num_memory_heads: int = 8
    num_memory_layers: int = 3
    num_seed_layers: int = 3
    target_vocab_size: int = 128256
    draft_vocab_size: int = 32000
    rms_norm_eps: float = 1e-5
    fusion_mode: str = "scalar"

    def __post_init__(self) -> None:
        sizes = (self.target_hidden_size, self.intermediate_size, self.num_memory_layers, self.num_seed_layers,
                 self.target_vocab_size, self.draft_vocab_size, self.num_memory_heads, self.head_dim)
        problems = [message for failed, message in (
            (self.num_attention_heads * self.head_dim != self.hidden_size,
             "hidden_size must equal num_attention_heads * head_dim"),
            (self.num_key_value_heads <= 0 or self.num_attention_heads % self.num_key_value_heads != 0,
             "num_attention_heads must be a multiple of num_key_value_heads"),
            (any(v <= 0 for v in sizes), "every architecture size must be positive"),
            (self.fusion_mode not in FUSION_MODES, f"fusion_mode must be one of {sorted(FUSION_MODES)}"),
        ) if failed]
        if problems:
            raise ValueError("; ".join(problems))

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> "SparseKVEagleConfig":
        return cls(**payload)


class EagleSelfAttention(nn.Module):
    """GQA attention of one new position over the recurrent per-position KV."""

    def __init__(self, config: SparseKVEagleConfig) -> None:
        super().__init__()
        width_in = 2 * config.hidden_size
        self.num_heads = config.num_attention_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.head_dim = config.head_dim
        self.q_proj = nn.Linear(width_in, self.num_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(width_in, self.num_key_value_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(width_in, self.num_key_value_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, config.hidden_size, bias=False)

    def forward(self, hidden, cos, sin, past_key, past_value):
        """``hidden`` [B, 1, 2H]; cos/sin [1, D] or [B, 1, D]; past K/V [B, Hkv, p, D] or None."""
        b, t, _ = hidden.shape
        if t != 1 or cos.shape[-2:] != (1, self.head_dim):
            raise ValueError("recurrent EAGLE attention expects exactly one position")
        q = self.q_proj(hidden).view(b, 1, self.num_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(hidden).view(b, 1, self.num_key_value_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(hidden).view(b, 1, self.num_key_value_heads, self.head_dim).transpose(1, 2)
        q = apply_rope(q, cos, sin, sequence_dim=2)
        k = apply_rope(k, cos, sin, sequence_dim=2)
        if past_key is not None:
            if past_value is None:
                raise ValueError("EAGLE key/value cache is incomplete")
            k = torch.cat((past_key, k), dim=2)
            v = torch.cat((past_value, v), dim=2)
        # one new position over every past one (GQA without repeating K/V):
        # this package's forward / backward kernels on CUDA, SDPA otherwise
        out = recurrent_attention(q, k, v).reshape(b, 1, self.num_heads * self.head_dim)
        return self.o_proj(out), k, v


class EagleMLP(nn.Module):
    def __init__(self, config: SparseKVEagleConfig) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=False)

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(hidden)) * self.up_proj(hidden))


class EagleDraftLayer(nn.Module):
    def __init__(self, config: SparseKVEagleConfig) -> None:
        super().__init__()
        self.self_attn = EagleSelfAttention(config)
        self.mlp = EagleMLP(config)
        self.hidden_norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)

    def forward(self, input_embedding, hidden, cos, sin, past_key, past_value):
        x = torch.cat((self.input_layernorm(input_embedding), self.hidden_norm(hidden)), dim=-1)
        attended, k, v = self.self_attn(x, cos, sin, past_key, past_value)
        hidden = hidden + attended
        hidden = hidden + self.mlp(self.post_attention_layernorm(hidden))
        return hidden, k, v


#: top-level modules and buffers of the EAGLE-3 trunk; everything else in the
#: drafter's state dict is the adapter, which an EAGLE-3 checkpoint lacks
EAGLE_TRUNK = frozenset({"midlayer", "fc", "norm", "lm_head", "d2t", "t2d"})


def vocab_maps(offsets: torch.Tensor, target_vocab: int) -> tuple[torch.Tensor, torch.Tensor]:
    """EAGLE's compressed vocabulary: draft id i is target id i + offsets[i].

    Returns (draft -> target ids, target -> draft ids with -1 for target ids
    outside the draft vocabulary); refuses a map that is not one-to-one.
    """
    n = offsets.numel()
    to_target = offsets.long() + torch.arange(n, device=offsets.device)
    if int(to_target.min()) < 0 or int(to_target.max()) >= target_vocab:
        raise ValueError("EAGLE compressed-vocabulary mapping leaves the target vocabulary")
    hits = torch.bincount(to_target, minlength=target_vocab)
    if int(hits.max()) > 1:
        raise ValueError("EAGLE compressed-vocabulary mapping is not one-to-one")
    to_draft = torch.full((target_vocab,), -1, dtype=torch.long, device=offsets.device)
    to_draft.scatter_(0, to_target, torch.arange(n, device=offsets.device))
    return to_target, to_draft


class SparseKVEagleDrafter(nn.Module):
    """Frozen EAGLE-3 proposal trunk plus a trainable sparse-target-KV adapter."""

    def __init__(self, config: SparseKVEagleConfig) -> None:
        super().__init__()
        self.config = config
        h = config.hidden_size
        self.midlayer = EagleDraftLayer(config)
        self.fc = nn.Linear(config.target_hidden_size * config.num_seed_layers, h, bias=False)
        self.norm = RMSNorm(h, config.rms_norm_eps)
        self.lm_head = nn.Linear(h, config.draft_vocab_size, bias=False)
        mem_cfg = SparseKVDraftConfig(
            target_hidden_size=config.target_hidden_size, draft_hidden_size=h, head_dim=config.head_dim,
            num_draft_heads=config.num_attention_heads, num_memory_heads=config.num_memory_heads,
            num_memory_layers=config.num_memory_layers, num_seed_layers=config.num_seed_layers,
            num_blocks=1, mlp_ratio=1, rms_norm_eps=config.rms_norm_eps)
        self.memory_norm = RMSNorm(h, config.rms_norm_eps)
        self.memory_attention = SparseTargetKVAttention(mem_cfg)
        # gated-delta fusion starts closed (gate bias -1, zero weights) with an identity delta map
        self.memory_gate = nn.Linear(3 * h, h)
        self.memory_delta = nn.Linear(h, h)
        with torch.no_grad():
            self.memory_gate.weight.zero_()
            self.memory_gate.bias.fill_(-1.0)
            self.memory_delta.weight.copy_(torch.eye(h))
            self.memory_delta.bias.zero_()
        if config.fusion_mode == "scalar":
            for p in (*self.memory_gate.parameters(), *self.memory_delta.parameters()):
                p.requires_grad_(False)
        self.adapter_scale = nn.Parameter(torch.tensor(-4.0))
        self.stage_layer_bias = nn.Linear(2, config.num_memory_layers, bias=True)
        with torch.no_grad():
            self.stage_layer_bias.weight.zero_()
            self.stage_layer_bias.bias.zero_()
        self.register_buffer("d2t", torch.zeros(config.draft_vocab_size, dtype=torch.long))
        self.register_buffer("t2d", torch.zeros(config.target_vocab_size, dtype=torch.bool))
        self.register_buffer("draft_to_target", torch.arange(config.draft_vocab_size, dtype=torch.long))
        self.register_buffer("target_to_draft", torch.full((config.target_vocab_size,), -1, dtype=torch.long))
        object.__setattr__(self, "_target_embedding_weight", None)

    # ---------------------------------------------------------------- binding
    def bind_target_embedding(self, embedding_weight: torch.Tensor) -> None:
        expected = (self.config.target_vocab_size, self.config.target_hidden_size)
        if tuple(embedding_weight.shape) != expected:
            raise ValueError("target embedding shape is incompatible with EAGLE")
        object.__setattr__(self, "_target_embedding_weight", embedding_weight.detach())

    def adapter_names(self) -> set[str]:
        """State-dict entries outside the EAGLE-3 trunk (the sparse-KV adapter)."""
        return {name for name in self.state_dict() if name.split(".", 1)[0] not in EAGLE_TRUNK}

    def load_eagle_checkpoint(self, checkpoint_path: str | Path) -> None:
        """Load an EAGLE-3 checkpoint: exactly the trunk, nothing more, nothing less."""
        state = torch.load(checkpoint_path, map_location="cpu", weights_only=True)
        result = self.load_state_dict(state, strict=False)
        if set(result.missing_keys) != self.adapter_names() or result.unexpected_keys:
            raise ValueError(f"incompatible EAGLE checkpoint: missing={result.missing_keys}, "
                             f"unexpected={result.unexpected_keys}")
        self._rebuild_vocab_maps()

    def _rebuild_vocab_maps(self) -> None:
        to_target, to_draft = vocab_maps(self.d2t, self.config.target_vocab_size)
        self.draft_to_target.copy_(to_target)
        self.target_to_draft.copy_(to_draft)

    def freeze_eagle(self) -> None:
        for module in (self.midlayer, self.fc, self.norm, self.lm_head):
            for p in module.parameters():
                p.requires_grad_(False)

    def adapter_parameters(self) -> list[nn.Parameter]:
        return [p for p in self.parameters() if p.requires_grad]

    def adapter_state_dict(self) -> dict[str, torch.Tensor]:
        """CPU copies of the trainable parameters (the adapter checkpoint payload)."""
        return {name: p.detach().cpu() for name, p in self.named_parameters() if p.requires_grad}

    def target_ids(self, draft_ids: torch.Tensor) -> torch.Tensor:
        return self.draft_to_target[draft_ids]

    def draft_ids(self, target_ids: torch.Tensor) -> torch.Tensor:
        return self.target_to_draft[target_ids]

    # ---------------------------------------------------------------- compute
    def fuse(self, hidden: torch.Tensor, delta: torch.Tensor) -> torch.Tensor:
        """What the memory read adds to the recurrent hidden state.

        scalar:       s * delta
        gated_delta:  s * g * W_d (delta - hidden),  g = sigmoid(W_g [hidden, delta, delta - hidden] + b_g)
        with s = sigmoid(adapter_scale).  These are the semantics trained
        adapters carry, so both implementations compute the same function.
        """
        s = torch.sigmoid(self.adapter_scale).to(hidden.dtype)
        if self.config.fusion_mode == "scalar":
            return s * delta
        toward = delta - hidden
        g = torch.sigmoid(self.memory_gate(torch.cat((hidden, delta, toward), dim=-1)))
        return s * g * self.memory_delta(toward)

    def _memory_delta(self, hidden, memory_keys, memory_values, cos, sin, stage) -> torch.Tensor:
        """Adapter output for the current position.  ``stage`` is [B, 2] (or [1, 2])."""
        layer_bias = self.stage_layer_bias(stage.float())  # [B, L]
        if layer_bias.shape[0] == 1:
            layer_bias = layer_bias[0]
        read = self.memory_attention(self.memory_norm(hidden), memory_keys, memory_values, cos, sin,
                                     layer_logits_bias=layer_bias)
        return self.fuse(hidden, read)

    def init_state(self, seed_hidden: torch.Tensor):
        """Recurrent state before the first draft position: (fc(seeds), no KV)."""
        b = seed_hidden.shape[0]
        return self.fc(seed_hidden.reshape(b, -1)).unsqueeze(1), None, None

    def step(self, token_ids: torch.Tensor, state, cos, sin, memory_keys, memory_values, stage,
             *, use_memory: bool = True):
        """One recurrent position for a batch: token_ids [B, 1] -> (normalised feature [B, 1, H], state)."""
        emb = self._target_embedding_weight
        if emb is None:
            raise RuntimeError("bind_target_embedding must be called before forward")
        hidden, past_k, past_v = state
        tok = F.embedding(token_ids, emb)
        hidden, past_k, past_v = self.midlayer(tok, hidden, cos, sin, past_k, past_v)
        if use_memory:
            hidden = hidden + self._memory_delta(hidden, memory_keys, memory_values, cos, sin, stage)
        return self.norm(hidden), (hidden, past_k, past_v)

    def recurrent_forward(
        self,
        input_ids: torch.Tensor,
        seed_hidden: torch.Tensor,
        memory_keys,
        memory_values,
        query_cos: torch.Tensor,
        query_sin: torch.Tensor,
        stage: torch.Tensor,
        *,
        use_memory: bool = True,
    ) -> torch.Tensor:
        """Normalised LM-head inputs [B, t, H] of every position.

        ``input_ids`` [B, t]; ``seed_hidden`` [B, seeds, target_hidden];
        ``query_cos``/``query_sin`` [t, D] (shared) or [B, t, D] (per row);
        ``stage`` [B, 2].  ``memory_keys`` is a [L, H, T, D] tensor shared by
        all rows (with ``memory_values``) or a per-row memory batch object.
        The LM head is left to the caller so that the logits of all positions
        can be formed in one GEMM (and fused with the loss).
        """
        if self._target_embedding_weight is None:
            raise RuntimeError("bind_target_embedding must be called before forward")
        state = self.init_state(seed_hidden)
        feats = []
        for p in range(input_ids.shape[1]):
            f, state = self.step(input_ids[:, p:p + 1], state, query_cos[..., p:p + 1, :],
                                 query_sin[..., p:p + 1, :], memory_keys, memory_values, stage,
                                 use_memory=use_memory)
            feats.append(f)
        return torch.cat(feats, dim=1)

    @torch.no_grad()
    def propose(self, first_token: torch.Tensor, seed_hidden, memory_keys, memory_values, query_cos, query_sin,
                stage, *, n_tokens: int, use_memory: bool = True) -> torch.Tensor:
        """Greedy draft of ``n_tokens`` target ids per row, feeding each proposal back.

        ``first_token`` [B, 1] is the last verified token; cos/sin cover the
        ``n_tokens`` positions ([n, D] or [B, n, D]).  Equals the reference's
        evaluation loop, which re-runs the prefix for every proposal.
        """
        state = self.init_state(seed_hidden)
        tok = first_token
        out = []
        for p in range(n_tokens):
            f, state = self.step(tok, state, query_cos[..., p:p + 1, :], query_sin[..., p:p + 1, :], memory_keys,
                                 memory_values, stage, use_memory=use_memory)
            draft = self.lm_head(f).argmax(-1)  # [B, 1]
            tok = self.target_ids(draft)
            out.append(tok)
        return torch.cat(out, dim=1)

    def forward(
        self,
        input_ids: torch.Tensor,
        seed_hidden: torch.Tensor,
        memory_keys: torch.Tensor,
        memory_values: torch.Tensor,
        query_cos: torch.Tensor,
        query_sin: torch.Tensor,
        *,
        visible_fraction: float,
        prompt_tokens: int,
        use_memory: bool = True,
        return_features: bool = False,
    ):
        cfg = self.config
        if self._target_embedding_weight is None:
            raise RuntimeError("bind_target_embedding must be called before forward")
        if input_ids.ndim != 2 or input_ids.shape[0] != 1:
            raise ValueError("sparse EAGLE currently requires batch size one")
        if tuple(seed_hidden.shape) != (1, cfg.num_seed_layers, cfg.target_hidden_size):
            raise ValueError("seed hidden-state shape is incompatible")
        t = input_ids.shape[1]
        if tuple(query_cos.shape) != (t, cfg.head_dim):
            raise ValueError("query RoPE shape does not match input tokens")
        if query_sin.shape != query_cos.shape:
            raise ValueError("query RoPE cosine/sine shapes differ")
        if not 0.0 < visible_fraction <= 1.0 or prompt_tokens <= 0:
            raise ValueError("invalid sparse-KV stage metadata")
        stage = stage_features(visible_fraction, prompt_tokens, dtype=torch.float32, device=input_ids.device)
        feats = self.recurrent_forward(input_ids, seed_hidden, memory_keys, memory_values, query_cos, query_sin,
                                       stage, use_memory=use_memory)
        logits = self.lm_head(feats)
        return (logits, feats) if return_features else logits
