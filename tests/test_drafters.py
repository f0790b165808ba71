"""Sparse-KV drafters: shapes, gradients, checkpoint scope, page selection
(behaviours of the reference's tests/test_sparse_kv_draft.py and
tests/test_sparse_kv_eagle.py), plus the batched recurrence and memory
batches this package adds."""
from pathlib import Path

import pytest
import torch

from sparsecache_b200.models.sparse_kv_draft import (
    SparseKVDraftConfig,
    SparseKVDrafter,
    accepted_prefix_length,
    select_visible_token_indices,
    sink_recent_topk_indices,
)
from sparsecache_b200.models.sparse_kv_eagle import SparseKVEagleConfig, SparseKVEagleDrafter
from sparsecache_b200.ops.sparse_attention import MemoryBatch


def _draft_cfg(**kw):
    base = dict(target_hidden_size=32, draft_hidden_size=16, head_dim=4, num_draft_heads=4, num_memory_heads=4,
                num_memory_layers=2, num_seed_layers=2, mlp_ratio=2)
    base.update(kw)
    return SparseKVDraftConfig(**base)


def test_drafter_forward_backward_and_state_excludes_target_weights():
    torch.manual_seed(0)
    model = SparseKVDrafter(_draft_cfg())
    model.bind_target_weights(torch.randn(64, 32), torch.randn(64, 32))
    logits = model(torch.tensor([[1, 2, 3]]), torch.randn(1, 2, 32), torch.randn(2, 4, 7, 4), torch.randn(2, 4, 7, 4),
                   torch.randn(3, 4), torch.randn(3, 4), visible_fraction=0.25, prompt_tokens=32)
    assert logits.shape == (1, 3, 64)
    assert all("target_" not in name for name in model.state_dict())
    logits.sum().backward()
    assert model.blocks[0].memory_attention.query[0].weight.grad is not None


def test_drafter_returns_target_space_features():
    cfg = _draft_cfg(target_hidden_size=16, draft_hidden_size=8, num_draft_heads=2, num_memory_heads=2,
                     num_memory_layers=1, num_seed_layers=1)
    model = SparseKVDrafter(cfg)
    model.bind_target_weights(torch.randn(20, 16), torch.randn(20, 16))
    logits, feats = model(torch.tensor([[1, 2]]), torch.randn(1, 1, 16), torch.randn(1, 2, 5, 4),
                          torch.randn(1, 2, 5, 4), torch.randn(2, 4), torch.randn(2, 4), visible_fraction=0.2,
                          prompt_tokens=10, return_features=True)
    assert logits.shape == (1, 2, 20) and feats.shape == (1, 2, 16)


def test_page_selection_protects_boundaries_deterministic_sorted():
    a = select_visible_token_indices(1000, page_size=64, visible_fraction=0.25, seed=7)
    b = select_visible_token_indices(1000, page_size=64, visible_fraction=0.25, seed=7)
    assert torch.equal(a, b)
    s = set(a.tolist())
    assert set(range(64)) <= s and set(range(960, 1000)) <= s
    assert torch.all(a[1:] > a[:-1])


def test_full_visibility_and_accepted_prefix():
    idx = select_visible_token_indices(130, page_size=64, visible_fraction=1.0, seed=0, mode="strided")
    assert idx.tolist() == list(range(130))
    assert accepted_prefix_length([1, 2, 9], [1, 2, 3]) == 2
    assert accepted_prefix_length([1], [1, 2]) == 1


def test_random_views_nest_for_one_seed():
    views = [set(select_visible_token_indices(4096, page_size=64, visible_fraction=f, seed=17).tolist())
             for f in (0.05, 0.10, 0.20)]
    assert views[0] < views[1] < views[2]


def test_priority_selection_takes_highest_unprotected_pages():
    sel = select_visible_token_indices(640, page_size=64, visible_fraction=0.3, seed=0, mode="priority",
                                       page_scores=torch.arange(10, dtype=torch.float32))
    assert {t // 64 for t in sel.tolist()} == {0, 8, 9}


def test_sink_recent_topk_view():
    T = 16384
    scores = torch.zeros(T // 64)
    scores[[10, 20, 30]] = torch.tensor([3.0, 2.0, 1.0])
    idx = sink_recent_topk_indices(T, scores)
    assert idx.numel() == 2048
    s = set(idx.tolist())
    assert set(range(64)) <= s and set(range(T - 512, T)) <= s
    assert set(range(640, 704)) <= s and set(range(1280, 1344)) <= s
    assert torch.all(idx[1:] > idx[:-1])
    assert sink_recent_topk_indices(1000, None).tolist() == list(range(1000))


def _eagle_cfg(**kw):
    base = dict(target_hidden_size=16, hidden_size=16, intermediate_size=32, head_dim=4, num_attention_heads=4,
                num_key_value_heads=2, num_memory_heads=2, num_memory_layers=2, num_seed_layers=2,
                target_vocab_size=32, draft_vocab_size=16, rms_norm_eps=1e-5)
    base.update(kw)
    return SparseKVEagleConfig(**base)


def test_eagle_forward_and_adapter_only_gradients():
    model = SparseKVEagleDrafter(_eagle_cfg())
    model.bind_target_embedding(torch.randn(32, 16))
    model.freeze_eagle()
    logits = model(torch.tensor([[1, 2, 3]]), torch.randn(1, 2, 16), torch.randn(2, 2, 7, 4), torch.randn(2, 2, 7, 4),
                   torch.randn(3, 4), torch.randn(3, 4), visible_fraction=0.25, prompt_tokens=64)
    assert logits.shape == (1, 3, 16)
    logits.sum().backward()
    assert model.memory_attention.query[0].weight.grad is not None
    assert model.midlayer.self_attn.q_proj.weight.grad is None


def test_eagle_memory_disabled_is_exactly_memory_independent():
    model = SparseKVEagleDrafter(_eagle_cfg())
    model.bind_target_embedding(torch.randn(32, 16))
    args = [torch.tensor([[1, 2]]), torch.randn(1, 2, 16), torch.randn(2, 2, 5, 4), torch.randn(2, 2, 5, 4),
            torch.randn(2, 4), torch.randn(2, 4)]
    a = model(*args, visible_fraction=0.1, prompt_tokens=32, use_memory=False)
    args[2] = torch.randn_like(args[2])
    b = model(*args, visible_fraction=0.1, prompt_tokens=32, use_memory=False)
    assert torch.equal(a, b)


def test_eagle_checkpoint_vocab_maps_and_adapter_state(tmp_path: Path):
    src = SparseKVEagleDrafter(_eagle_cfg())
    state = {n: t for n, t in src.state_dict().items()
             if not n.startswith(("memory_", "stage_")) and n not in {"adapter_scale", "draft_to_target",
                                                                       "target_to_draft"}}
    state["d2t"] = torch.arange(16)
    state["t2d"] = torch.zeros(32, dtype=torch.bool)
    ckpt = tmp_path / "eagle.pt"
    torch.save(state, ckpt)
    model = SparseKVEagleDrafter(_eagle_cfg())
    model.load_eagle_checkpoint(ckpt)
    model.freeze_eagle()
    assert model.draft_to_target.tolist() == list(range(0, 32, 2))
    assert model.draft_ids(torch.tensor([0, 2, 31])).tolist() == [0, 1, -1]
    adapter = model.adapter_state_dict()
    assert adapter and all(n.startswith(("memory_", "stage_")) or n == "adapter_scale" for n in adapter)
    # an unexpected tensor is refused
    state["bogus"] = torch.zeros(1)
    torch.save(state, ckpt)
    try:
        SparseKVEagleDrafter(_eagle_cfg()).load_eagle_checkpoint(ckpt)
    except ValueError:
        pass
    else:
        raise AssertionError("an unexpected tensor must be rejected")


def test_gated_delta_gradients_reach_gate_and_delta():
    model = SparseKVEagleDrafter(_eagle_cfg(fusion_mode="gated_delta"))
    model.bind_target_embedding(torch.randn(32, 16))
    logits = model(torch.tensor([[1, 2]]), torch.randn(1, 2, 16), torch.randn(2, 2, 5, 4), torch.randn(2, 2, 5, 4),
                   torch.randn(2, 4), torch.randn(2, 4), visible_fraction=0.2, prompt_tokens=32)
    logits.sum().backward()
    assert model.memory_gate.weight.grad is not None and model.memory_delta.weight.grad is not None


def test_batched_recurrence_with_memory_batch_matches_per_row_forward():
    """Rows of one batched recurrence (own memory, positions and stage each)
    equal the batch-1 forward of each row."""
    torch.manual_seed(1)
    cfg = _eagle_cfg(head_dim=4)
    model = SparseKVEagleDrafter(cfg)
    model.bind_target_embedding(torch.randn(32, 16))
    with torch.no_grad():
        model.adapter_scale.fill_(0.5)
        model.stage_layer_bias.weight.normal_()
    S, L, T, H, D = 3, 2, 9, 2, 4
    keys, values = torch.randn(S, L, T, H, D), torch.randn(S, L, T, H, D)
    n_vis = torch.tensor([9, 5, 7], dtype=torch.int32)
    idx = torch.stack([torch.randperm(T)[:T].sort().values for _ in range(S)]).to(torch.int32)
    row_seq = torch.tensor([2, 0], dtype=torch.int32)
    mem = MemoryBatch(keys, values, idx, n_vis, row_seq)
    ids = torch.tensor([[1, 4, 7], [3, 3, 9]])
    seeds = torch.randn(2, 2, 16)
    cos, sin = torch.randn(2, 3, 4), torch.randn(2, 3, 4)
    stage = torch.tensor([[0.3, 0.5], [0.7, 0.2]])
    feats = model.recurrent_forward(ids, seeds, mem, None, cos, sin, stage)
    for b in range(2):
        s = int(row_seq[b])
        sel = idx[s, : n_vis[s]].long()
        k = keys[s, :, sel].permute(0, 2, 1, 3)  # [L, H, n, D]
        v = values[s, :, sel].permute(0, 2, 1, 3)
        ref = model.recurrent_forward(ids[b:b + 1], seeds[b:b + 1], k, v, cos[b], sin[b], stage[b:b + 1])
        assert torch.allclose(feats[b], ref[0], atol=2e-5), (b, (feats[b] - ref[0]).abs().max())


def test_propose_matches_reference_style_prefix_rerun():
    torch.manual_seed(2)
    model = SparseKVEagleDrafter(_eagle_cfg())
    model.bind_target_embedding(torch.randn(32, 16))
    seeds = torch.randn(1, 2, 16)
    k, v = torch.randn(2, 2, 6, 4), torch.randn(2, 2, 6, 4)
    cos, sin = torch.randn(4, 4), torch.randn(4, 4)
    stage = torch.tensor([[0.2, 0.4]])
    prop = model.propose(torch.tensor([[5]]), seeds, k, v, cos, sin, stage, n_tokens=4)[0].tolist()
    prefix = [5]
    for _ in range(4):
        logits = model.lm_head(model.recurrent_forward(torch.tensor([prefix]), seeds, k, v, cos[:len(prefix)],
                                                       sin[:len(prefix)], stage))
        prefix.append(int(model.target_ids(logits[0, -1].argmax())))
    assert prop == prefix[1:]


def test_tp_drafter_shards_reassemble_the_module():
    """Every rank's shard of the EAGLE drafter (heads, 128-row gate/up blocks, memory heads)
    concatenates back to the module's weights; replicated parts are identical."""
    import torch

    from sparsecache_b200.models.sparse_kv_eagle import SparseKVEagleConfig, SparseKVEagleDrafter
    from sparsecache_b200.models.weights import split_gate_up
    from sparsecache_b200.parallel.tp_draft import TPDraftWeights

    cfg = SparseKVEagleConfig(target_hidden_size=512, hidden_size=512, intermediate_size=1024, head_dim=128,
                              num_attention_heads=4, num_key_value_heads=2, num_memory_heads=2, num_memory_layers=3,
                              num_seed_layers=3, target_vocab_size=4096, draft_vocab_size=1024)
    torch.manual_seed(0)
    m = SparseKVEagleDrafter(cfg)
    tp = 2
    shards = [TPDraftWeights.from_module(m, r, tp, "cpu") for r in range(tp)]
    at, mlp = m.midlayer.self_attn, m.midlayer.mlp
    bf = lambda t: t.detach().to(torch.bfloat16)  # noqa: E731
    q = torch.cat([s.w_qkv[:2 * 128] for s in shards])
    k = torch.cat([s.w_qkv[2 * 128:3 * 128] for s in shards])
    v = torch.cat([s.w_qkv[3 * 128:] for s in shards])
    assert torch.equal(q, bf(at.q_proj.weight)) and torch.equal(k, bf(at.k_proj.weight))
    assert torch.equal(v, bf(at.v_proj.weight))
    assert torch.equal(torch.cat([s.w_o for s in shards], 1), bf(at.o_proj.weight))
    gates, ups = zip(*(split_gate_up(s.w_gu) for s in shards))
    assert torch.equal(torch.cat(gates), bf(mlp.gate_proj.weight)) and torch.equal(torch.cat(ups), bf(mlp.up_proj.weight))
    assert torch.equal(torch.cat([s.w_down for s in shards], 1), bf(mlp.down_proj.weight))
    for i in range(3):
        qi = torch.cat([s.w_memq[i * 128:(i + 1) * 128] for s in shards])
        assert torch.equal(qi, bf(m.memory_attention.query[i].weight))
        assert torch.equal(torch.cat([s.w_memo[i] for s in shards], 1), bf(m.memory_attention.output[i].weight))
    assert all(torch.equal(s.lm_head, shards[0].lm_head) and torch.equal(s.fc, shards[0].fc) for s in shards)
    assert shards[0].d2t.dtype == torch.int32 and abs(shards[0].adapter_scale - torch.sigmoid(torch.tensor(-4.0)).item()) < 1e-6
    import pytest

    with pytest.raises(ValueError):
        TPDraftWeights.from_module(m, 0, 3, "cpu")


def test_eagle_adapter_names_and_vocab_rules():
    """The adapter (what an EAGLE-3 checkpoint lacks) is exactly this set of
    names, for any number of memory layers; the vocabulary map must stay in
    range and be one-to-one."""
    from sparsecache_b200.models.sparse_kv_eagle import vocab_maps

    for layers in (1, 3):
        cfg = SparseKVEagleConfig(**{**_eagle_cfg().to_dict(), "num_memory_layers": layers})
        names = SparseKVEagleDrafter(cfg).adapter_names()
        expect = {"adapter_scale", "draft_to_target", "target_to_draft", "memory_norm.weight",
                  "memory_attention.layer_gates", "stage_layer_bias.weight", "stage_layer_bias.bias",
                  "memory_gate.weight", "memory_gate.bias", "memory_delta.weight", "memory_delta.bias"}
        expect |= {f"memory_attention.{k}.{i}.weight" for k in ("query", "output") for i in range(layers)}
        assert names == expect
    to_t, to_d = vocab_maps(torch.tensor([0, 1, 1, 5]), 10)
    assert to_t.tolist() == [0, 2, 3, 8] and to_d.tolist() == [0, -1, 1, 2, -1, -1, -1, -1, 3, -1]
    with pytest.raises(ValueError, match="one-to-one"):
        vocab_maps(torch.tensor([1, 0]), 4)
    with pytest.raises(ValueError, match="target vocabulary"):
        vocab_maps(torch.tensor([0, 9]), 4)
    with pytest.raises(ValueError, match="multiple of num_key_value_heads"):
        SparseKVEagleConfig(**{**_eagle_cfg().to_dict(), "num_key_value_heads": 3})
