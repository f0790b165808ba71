"""Tensor-parallel sparse-KV EAGLE drafter and speculative decoding on the decode GEMV kernels.

Serving-side counterpart of ``models.sparse_kv_eagle.SparseKVEagleDrafter``
(the reference's EAGLE-3 trunk + sparse target-KV adapter,
experiments/train_sparse_kv_eagle.py:97-175 for the losses and
src/sparsecache/sparse_kv_eagle.py for the module; the verify/accept protocol
follows experiments/progressive_kv_feasibility.py:616-682 and
experiments/reuse_cacheblend_pipeline.py:782-825).  One draft position is

    x  = [rmsnorm_in(embed(token)), rmsnorm_hidden(hidden)]          (2 d)
    h  = hidden + o(attn(qkv(x)))           self-attention over this proposal's positions
    h  = h + down(swiglu(gate_up(rmsnorm_post(h))))
    h  = h + s * sum_i g_i * out_i(attn_i(q_i(rmsnorm_mem(h)), target layer i, sparse view))
    draft = argmax(lm_head(rmsnorm(h)))  ->  target id (draft-to-target map)

with the first hidden = fc(seed features of 3 target layers).  Under tensor
parallelism the drafter is sharded like the target: the self-attention and
memory heads by head (memory head h reads the target's kv head h, which is
local), gate/up by 128-row blocks, and o / down / memory-out are row-parallel
GEMVs whose partials are all-reduced inside the GEMV kernel over peer
memory (``TPEngine.allreduce``).  fc, the norms and the draft LM head are
replicated.  The layer gates g_i = softmax(layer_gates + stage_bias(stage))
and the adapter scale s are constant for a request, so they are folded into
the memory output weights once per request.

A proposal of gamma tokens is one CUDA graph (3 * gamma all-reduces; gamma
even keeps the two receive buffers alternating); ``speculative_generate``
alternates it with the target's batched verify step and accepts the longest
matching prefix plus the target's token after it.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..models.weights import GATE_UP_BLOCK, interleave_gate_up
from .tp import TPEngine


@dataclass
class TPDraftWeights:
    """One rank's drafter weights (bf16 unless noted)."""

    fc: torch.Tensor            # [d, n_seed * d_target] replicated
    in_ln: torch.Tensor
    hid_ln: torch.Tensor
    w_qkv: torch.Tensor         # [(hq + 2 hkv) * 128, 2 d] this rank's heads
    w_o: torch.Tensor           # [d, hq * 128]
    post_ln: torch.Tensor
    w_gu: torch.Tensor          # [2 f, d], gate/up interleaved in 128-row blocks
    w_down: torch.Tensor        # [d, f]
    mem_ln: torch.Tensor
    w_memq: torch.Tensor        # [n_mem * hm * 128, d] this rank's memory heads, layer-major
    w_memo: list[torch.Tensor]  # n_mem x [d, hm * 128]
    layer_gates: torch.Tensor   # [n_mem] fp32
    stage_w: torch.Tensor       # [n_mem, 2] fp32
    stage_b: torch.Tensor       # [n_mem] fp32
    adapter_scale: float
    norm: torch.Tensor
    lm_head: torch.Tensor       # [V_draft, d] replicated
    d2t: torch.Tensor           # [V_draft] int32 target ids

    @staticmethod
    def _heads(w: torch.Tensor, first: int, count: int) -> torch.Tensor:
        return w[first * 128:(first + count) * 128]

    @classmethod
    def from_module(cls, model, rank: int, tp: int, device) -> "TPDraftWeights":
        """This rank's shard of a ``SparseKVEagleDrafter`` (scalar fusion mode)."""
        c = model.config
        if c.fusion_mode != "scalar":
            raise ValueError("the serving drafter implements the scalar fusion mode")
        if c.num_attention_heads % tp or c.num_key_value_heads % tp or c.num_memory_heads % tp \
                or c.intermediate_size % (tp * GATE_UP_BLOCK):
            raise ValueError("drafter heads / ffn do not divide by the TP size")
        bf = torch.bfloat16
        hq, hkv, hm, f = (c.num_attention_heads // tp, c.num_key_value_heads // tp, c.num_memory_heads // tp,
                          c.intermediate_size // tp)
        ml = model.midlayer
        at = ml.self_attn

        def t(x):
            return x.detach().to(device=device, dtype=bf).contiguous()

        qkv = torch.cat((cls._heads(at.q_proj.weight, rank * hq, hq), cls._heads(at.k_proj.weight, rank * hkv, hkv),
                         cls._heads(at.v_proj.weight, rank * hkv, hkv)))
        gate = ml.mlp.gate_proj.weight[rank * f:(rank + 1) * f]
        up = ml.mlp.up_proj.weight[rank * f:(rank + 1) * f]
        ma = model.memory_attention
        memq = torch.cat([cls._heads(q.weight, rank * hm, hm) for q in ma.query])
        memo = [t(o.weight[:, rank * hm * 128:(rank + 1) * hm * 128]) for o in ma.output]
        f32 = dict(device=device, dtype=torch.float32)
        return cls(fc=t(model.fc.weight), in_ln=t(ml.input_layernorm.weight), hid_ln=t(ml.hidden_norm.weight),
                   w_qkv=t(qkv), w_o=t(at.o_proj.weight[:, rank * hq * 128:(rank + 1) * hq * 128]),
                   post_ln=t(ml.post_attention_layernorm.weight), w_gu=t(interleave_gate_up(gate, up)),
                   w_down=t(ml.mlp.down_proj.weight[:, rank * f:(rank + 1) * f]), mem_ln=t(model.memory_norm.weight),
                   w_memq=t(memq), w_memo=memo, layer_gates=ma.layer_gates.detach().to(**f32),
                   stage_w=model.stage_layer_bias.weight.detach().to(**f32),
                   stage_b=model.stage_layer_bias.bias.detach().to(**f32),
                   adapter_scale=float(torch.sigmoid(model.adapter_scale.detach().float())),
                   norm=t(model.norm.weight), lm_head=t(model.lm_head.weight),
                   d2t=model.draft_to_target.detach().to(device=device, dtype=torch.int32))

    @classmethod
    def random(cls, c, rank: int, tp: int, seed: int, device) -> "TPDraftWeights":
        """Seeded random shard of a drafter of config ``c`` (no full-model materialisation)."""
        from .tp_bench import stable_seed

        bf = torch.bfloat16
        gen = torch.Generator(device=device)
        hq, hkv, hm, f = (c.num_attention_heads // tp, c.num_key_value_heads // tp, c.num_memory_heads // tp,
                          c.intermediate_size // tp)
        h = c.hidden_size

        def mat(rows, cols, tag, replicated=False):
            gen.manual_seed(stable_seed(seed, tag) if replicated else stable_seed(seed, tag, rank))
            return torch.empty(rows, cols, device=device, dtype=bf).normal_(0.0, 0.02, generator=gen)

        ones = torch.ones(h, device=device, dtype=bf)
        n = c.num_memory_layers
        f32 = dict(device=device, dtype=torch.float32)
        return cls(fc=mat(h, c.num_seed_layers * c.target_hidden_size, "fc", True), in_ln=ones, hid_ln=ones,
                   w_qkv=mat((hq + 2 * hkv) * 128, 2 * h, "qkv"), w_o=mat(h, hq * 128, "o"), post_ln=ones,
                   w_gu=mat(2 * f, h, "gu"), w_down=mat(h, f, "down"), mem_ln=ones,
                   w_memq=mat(n * hm * 128, h, "memq"), w_memo=[mat(h, hm * 128, ("memo", i)) for i in range(n)],
                   layer_gates=torch.zeros(n, **f32), stage_w=torch.zeros(n, 2, **f32), stage_b=torch.zeros(n, **f32),
                   adapter_scale=float(torch.sigmoid(torch.tensor(-4.0))), norm=ones,
                   lm_head=mat(c.draft_vocab_size, h, "lm_head", True),
                   d2t=torch.arange(c.draft_vocab_size, device=device, dtype=torch.int32))


class TPEagleDrafter:
    """Graph-captured gamma-token proposals on a ``TPEngine``'s group and kernels."""

    def __init__(self, tpe: TPEngine, config, weights: TPDraftWeights, *, memory_layers, gamma: int = 4,
                 view_capacity: int = 8192) -> None:
        if gamma < 1 or gamma % 2:
            raise ValueError("gamma must be even (the proposal graph alternates the all-reduce buffers)")
        if len(memory_layers) != config.num_memory_layers:
            raise ValueError("one target layer per memory layer")
        self.tpe, self.c, self.w = tpe, config, weights
        self.memory_layers = tuple(int(x) for x in memory_layers)
        self.gamma = gamma
        eng = tpe.engine
        dev = eng.device
        tp = tpe.tp
        c = config
        self.hq, self.hkv, self.hm = c.num_attention_heads // tp, c.num_key_value_heads // tp, c.num_memory_heads // tp
        if self.hm != tpe.lcfg.n_kv_heads:
            raise ValueError("memory heads must equal the target's kv heads (head h reads kv head h)")
        self.f = c.intermediate_size // tp
        h = c.hidden_size
        bf = torch.bfloat16
        z = lambda *s, dt=bf: torch.zeros(*s, device=dev, dtype=dt)  # noqa: E731
        self.seed = z(1, c.num_seed_layers * c.target_hidden_size)
        self.tok_in = z(1, dt=torch.int32)
        self.emb = z(1, c.target_hidden_size)
        self.hid = z(1, h)
        self.x2 = z(1, 2 * h)
        self.q = z(1, self.hq * 128)
        self.attn = z(1, self.hq * 128)
        self.act = z(1, self.f)
        mw = c.num_memory_layers * self.hm * 128
        self.mq = z(1, mw)
        self.ma = z(1, mw)
        self.dcap = 16
        self.dk = z(self.hkv, self.dcap, 128)
        self.dv = z(self.hkv, self.dcap, 128)
        self.dummy = z(1, 1, 128)
        self.dpos = z(gamma, dt=torch.int32)
        self.dslot = torch.arange(gamma, device=dev, dtype=torch.int32)
        self.nv = z(1, dt=torch.int32)
        self.view = z(view_capacity, dt=torch.int32)
        grid = eng.ext.gemv_argmax_grid(c.draft_vocab_size)
        self.pv = z(grid, dt=torch.float32)
        self.pi = z(grid, dt=torch.int32)
        self.counter = z(1, dt=torch.int32)
        self.dtok = z(gamma, dt=torch.int32)
        self.ttok = z(gamma, dt=torch.int32)
        self.memo = z(h, mw)
        self.scale = 1.0 / math.sqrt(128)
        self.n_visible = 0
        self.prompt_tokens = 0
        self._graph = None
        self._graph_key = None

    # ------------------------------------------------------------ request
    def set_request(self, visible: torch.Tensor, prompt_tokens: int, *, visible_fraction: float | None = None,
                    max_new: int = 1024) -> None:
        """Memory view of a request: sorted visible prompt indices (device int32), then the generated tail.

        Also folds this request's layer gates and adapter scale into the
        memory output weights.
        """
        n = int(visible.numel())
        T = int(prompt_tokens)
        if n + max_new + self.gamma + 1 > self.view.numel():
            raise ValueError("memory view exceeds its capacity")
        self.view[:n].copy_(visible.to(torch.int32))
        self.tpe.ext.arange_i32(self.view[n:n + max_new + self.gamma + 1], T)
        self.n_visible, self.prompt_tokens = n, T
        frac = n / max(1, T) if visible_fraction is None else float(visible_fraction)
        stage = torch.tensor([frac, math.log2(T + 1) / 17.0], device=self.w.stage_w.device)
        g = torch.softmax(self.w.layer_gates + self.w.stage_w @ stage + self.w.stage_b, dim=-1) * self.w.adapter_scale
        w = self.hm * 128
        for i, wo in enumerate(self.w.w_memo):
            self.memo[:, i * w:(i + 1) * w].copy_((wo.float() * g[i]).to(torch.bfloat16))

    # ------------------------------------------------------------- graph
    def _body(self, slot) -> None:
        tpe, w, c = self.tpe, self.w, self.c
        eng, ext = tpe.engine, tpe.ext
        b = eng._decode_buffers()
        eps = c.rms_norm_eps
        h = c.hidden_size
        d_splits = int(ext.attention_decode_cluster(self.dcap, self.hkv))
        m_splits = eng._decode_splits(slot.capacity)
        mw = self.hm * 128
        ext.gemv_store(self.seed, w.fc, None, eps, self.hid)
        for j in range(self.gamma):
            tok = self.tok_in if j == 0 else self.ttok[j - 1:j]
            ext.embedding(tok, eng.w.embed, self.emb)
            ext.rmsnorm(self.emb, None, w.in_ln, eps, self.x2[:, :h])
            ext.rmsnorm(self.hid, None, w.hid_ln, eps, self.x2[:, h:])
            ext.gemv_qkv(self.x2, w.w_qkv, None, eps, self.q, self.dk, self.dv, self.dpos[j:j + 1], eng.rope,
                         self.hq, self.hkv, slot=self.dslot[j:j + 1])
            ext.attention_decode(self.q, self.dk, self.dv, self.dslot[j:j + 1], self.hq, self.scale, d_splits,
                                 self.attn, ws=b["attn_ws"], counters=b["attn_cnt"])
            tpe.allreduce(self.attn, w.w_o, 3 * j + 1, self.hid)
            ext.gemv_swiglu(self.hid, w.w_gu, w.post_ln, eps, self.act)
            tpe.allreduce(self.act, w.w_down, 3 * j + 2, self.hid)
            ext.gemv_qkv(self.hid, w.w_memq, w.mem_ln, eps, self.mq, self.dummy, self.dummy, self.dpos[j:j + 1],
                         eng.rope, c.num_memory_layers * self.hm, 0, slot=self.dslot[j:j + 1])
            for i, layer in enumerate(self.memory_layers):
                ext.attention_decode(self.mq[:, i * mw:(i + 1) * mw], slot.k(layer), slot.v(layer), self.nv,
                                     self.hm, self.scale, m_splits, self.ma[:, i * mw:(i + 1) * mw],
                                     page_table=self.view, page_shift=0, n_virtual=self.nv, ws=b["attn_ws"],
                                     counters=b["attn_cnt"])
            tpe.allreduce(self.ma, self.memo, 3 * j + 3, self.hid)
            ext.gemv_argmax(self.hid, w.lm_head, w.norm, eps, self.pv, self.pi, self.counter, self.dtok[j:j + 1],
                            None, None, None, None, None)
            torch.index_select(w.d2t, 0, self.dtok[j:j + 1], out=self.ttok[j:j + 1])
        ext.bump_counter(b["pos"][3:4])

    def launches_per_proposal(self) -> int:
        """Kernels of this package per proposal (the index_select map is a torch op)."""
        return 1 + self.gamma * (14 + len(self.memory_layers)) + 1

    def propose(self, slot, first_token: torch.Tensor, seed_row: torch.Tensor, position: int, *,
                use_graph: bool = True) -> torch.Tensor:
        """gamma target-id drafts after ``first_token`` (device int32 [1]) at ``position``.

        ``seed_row`` [n_seed, d_target] are the target's residual rows of the
        last verified position; target keys [0, position) are valid.
        """
        ext = self.tpe.ext
        self.seed.view(-1).copy_(seed_row.reshape(-1))
        self.tok_in.copy_(first_token.reshape(1))
        # scalars go in as kernel arguments (no pinned staging to race with)
        self.nv.fill_(self.n_visible + (int(position) - self.prompt_tokens))
        ext.arange_i32(self.dpos, int(position))
        if not use_graph:
            self._body(slot)
            return self.ttok
        key = id(slot)
        if self._graph is None or self._graph_key != key:
            saved = self.hid.clone()
            self._body(slot)  # warm step (launch attributes); the drafts are recomputed below
            self.hid.copy_(saved)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._body(slot)
            self._graph, self._graph_key = graph, key
        self._graph.replay()
        ext.launches += self.launches_per_proposal()
        return self.ttok


def speculative_generate(tpe: TPEngine, drafter: TPEagleDrafter | None, slot, *, prompt_tokens: int, max_new: int,
                         use_graph: bool = True, proposal_trace=None) -> dict:
    """Greedy generation from the state ``first_token`` left (token 0 in the log, position T).

    With a drafter: verify [last token] once (seed features), then repeat
    propose gamma -> verify gamma + 1 rows -> accept the longest prefix of
    drafts equal to the target's argmax plus the target's next token.  One
    host read per iteration.  Without a drafter every step verifies one row
    (plain greedy decoding through the verify path).  Returns the tokens
    (first token included), accepted drafts per iteration and step counts.
    ``proposal_trace``: a path that receives the first proposal (seed and
    draft ids, atomically, first writer wins) for trace verification.
    """
    import time

    from ..serving.live.trace import publish_proposal_trace

    eng = tpe.engine
    b = eng._decode_buffers()
    feat = eng.ws.get("tp_feat", (len(tpe.seed_layers), eng.MAX_ROWS, tpe.full_cfg.d_model), torch.bfloat16)
    rows = eng.ws.get("tp_spec_rows", (eng.MAX_ROWS,), torch.int32)
    first = int(b["log"][0].item())
    tokens = [first]
    P = int(prompt_tokens)
    rows[0:1].copy_(b["log"][0:1])
    pred = tpe.verify(slot, rows[0:1], P, use_graph=use_graph).tolist()
    tokens.append(pred[0])
    P += 1
    n_acc, accepted, verifies = 0, [], 1
    while len(tokens) < max_new:
        rows[0:1].copy_(b["tok"][n_acc:n_acc + 1])
        if drafter is None:
            pred = tpe.verify(slot, rows[0:1], P, use_graph=use_graph).tolist()
            n_acc = 0
            new = [pred[0]]
        else:
            g = drafter.gamma
            started_ns = time.time_ns()
            drafts = drafter.propose(slot, rows[0:1], feat[:, n_acc], P, use_graph=use_graph)
            rows[1:1 + g].copy_(drafts)
            pred = tpe.verify(slot, rows[:1 + g], P, use_graph=use_graph).tolist()
            d = rows[1:1 + g].tolist()
            if proposal_trace is not None and not accepted:
                publish_proposal_trace(proposal_trace, method="eagle3", proposal_started_at_ns=started_ns,
                                       seed_token_ids=[tokens[-1]], draft_token_ids=d)
            n_acc = 0
            while n_acc < g and d[n_acc] == pred[n_acc]:
                n_acc += 1
            new = d[:n_acc] + [pred[n_acc]]
            accepted.append(n_acc)
        verifies += 1
        tpe.check_status()  # the host read above synchronised: a timed-out wait surfaces here
        tokens.extend(new)
        P += len(new)
    return {"tokens": tokens[:max_new], "accepted": accepted, "verify_steps": verifies,
            "mean_accepted": (sum(accepted) / len(accepted)) if accepted else 0.0}
