"""Drafter trainer on CPU: losses, flat trainables, AdamW oracle, step loop,
checkpoint/resume, evaluation (the reference's trainer tests exercise the
same behaviours through experiments/train_sparse_kv_*.py)."""
import math
from pathlib import Path

import torch

from sparsecache_b200.models.sparse_kv_eagle import SparseKVEagleConfig, SparseKVEagleDrafter
from sparsecache_b200.training.drafter_trainer import (
    DrafterTrainConfig,
    EagleDrafterTrainer,
    FlatTrainables,
    FusedAdamW,
    configure_trainable_modules,
    evaluate_drafter,
    load_adapter_checkpoint,
    random_eagle_drafter,
)
from sparsecache_b200.training.losses import (
    compressed_distillation_loss,
    feature_distillation_loss,
    prefix_weights,
    target_sequence_score,
    weighted_distillation_loss,
)
from sparsecache_b200.training.teacher import synthetic_bank


def _cfg(**kw):
    base = dict(target_hidden_size=16, hidden_size=16, intermediate_size=32, head_dim=8, num_attention_heads=2,
                num_key_value_heads=1, num_memory_heads=2, num_memory_layers=2, num_seed_layers=2,
                target_vocab_size=40, draft_vocab_size=24, rms_norm_eps=1e-5)
    base.update(kw)
    return SparseKVEagleConfig(**base)


def test_prefix_weights_and_weighted_loss_values():
    w = prefix_weights(3, prefix_decay=0.5)
    assert torch.allclose(w, torch.tensor([4.0, 2.0, 1.0]) / 7.0)
    logits = torch.zeros(1, 3, 5)
    labels = torch.tensor([0, 1, 2])
    ids = torch.tensor([[0, 1], [1, 2], [2, 3]])
    lps = torch.zeros(3, 2)
    loss, comps = weighted_distillation_loss(logits, labels, ids, lps, prefix_decay=0.9, hard_weight=1.0,
                                             soft_weight=0.5)
    assert math.isclose(float(comps["hard_loss"]), math.log(5), rel_tol=1e-6)
    assert math.isclose(float(loss), 1.5 * math.log(5), rel_tol=1e-6)


def test_feature_loss_and_sequence_score():
    f = torch.randn(1, 4, 8)
    assert float(feature_distillation_loss(f, f[0].clone(), prefix_decay=0.9)) < 1e-6
    assert float(feature_distillation_loss(f, -f[0], prefix_decay=0.9)) > 1.99
    logits = torch.randn(1, 4, 10)
    labels = torch.tensor([1, 2, 3, 4])
    s = target_sequence_score(logits, labels, prefix_decay=0.9)
    lp = logits.log_softmax(-1)[0, torch.arange(4), labels]
    assert torch.allclose(s, (lp * prefix_weights(4, prefix_decay=0.9)).sum())


def test_compressed_loss_skips_unmapped_labels():
    model = SparseKVEagleDrafter(_cfg(target_vocab_size=32, draft_vocab_size=16))
    model.target_to_draft[20] = 0
    logits = torch.randn(1, 2, 16, requires_grad=True)
    loss, comps = compressed_distillation_loss(model, logits, torch.tensor([21, 21]),
                                               torch.tensor([[20, 21], [20, 21]]), torch.zeros(2, 2),
                                               prefix_decay=0.9, hard_weight=1.0, soft_weight=0.5)
    assert float(comps["label_coverage"]) == 0.0 and float(comps["topk_coverage"]) == 0.5
    loss.backward()
    assert logits.grad is not None and torch.isfinite(logits.grad).all()


def test_flat_trainables_views_and_adamw_oracle_matches_torch():
    torch.manual_seed(0)
    a = torch.nn.Linear(5, 3)
    b = torch.nn.Linear(5, 3)
    b.load_state_dict(a.state_dict())
    flat = FlatTrainables(list(a.parameters()), device="cpu")
    assert a.weight.data_ptr() == flat.param.data_ptr()
    cfg = DrafterTrainConfig(lr=1e-2, weight_decay=0.1, grad_clip=0.05)
    opt = FusedAdamW(flat, cfg)
    ref = torch.optim.AdamW(b.parameters(), lr=1e-2, weight_decay=0.1)
    x = torch.randn(7, 5)
    for _ in range(3):
        flat.grad.zero_()
        a(x).square().sum().backward()
        opt.step()
        ref.zero_grad()
        b(x).square().sum().backward()
        torch.nn.utils.clip_grad_norm_(b.parameters(), 0.05)
        ref.step()
    assert torch.allclose(a.weight, b.weight, atol=1e-6) and torch.allclose(a.bias, b.bias, atol=1e-6)


def _trainer(tmp_batch=4):
    torch.manual_seed(0)
    cfg = _cfg()
    model = random_eagle_drafter(cfg, seed=0, std=0.2)
    model.bind_target_embedding(torch.randn(cfg.target_vocab_size, cfg.target_hidden_size))
    model.freeze_eagle()
    configure_trainable_modules(model, train_fc=False, train_midlayer=False, adapter_scale_init=0.0)
    bank = synthetic_bank(n_samples=8, horizon=5, n_layers=2, n_heads=2, n_seed=2, target_hidden=16, hidden=16,
                          vocab=24, visible=6, prompt_tokens=30, topk=4, device="cpu", head_dim=8)
    cos, sin = torch.randn(64, 8), torch.randn(64, 8)
    tcfg = DrafterTrainConfig(lr=3e-2, global_batch=tmp_batch, use_graph=False, feature_weight=0.5)
    return model, bank, cos, sin, EagleDrafterTrainer(model, bank, cos, sin, tcfg)


def test_trainer_steps_reduce_loss_and_only_adapter_moves():
    model, bank, cos, sin, tr = _trainer()
    trunk = model.midlayer.self_attn.q_proj.weight.detach().clone()
    losses = []
    for _ in range(12):
        tr.train_step()
        losses.append(float(tr.loss))
    assert losses[-1] < losses[0]
    assert torch.equal(trunk, model.midlayer.self_attn.q_proj.weight)
    row = tr.log_row()
    assert row["step"] == 12 and math.isfinite(row["grad_norm"])


def test_trainer_checkpoint_resume_roundtrip(tmp_path: Path):
    model, bank, cos, sin, tr = _trainer()
    for _ in range(3):
        tr.train_step()
    path = tmp_path / "adapter.pt"
    tr.save(path)
    model2, _, _, _, tr2 = _trainer()
    ckpt = tr2.resume(path)
    assert ckpt["completed_steps"] == 3 and tr2.steps_done == 3
    for (n, p), (_, q) in zip(model.named_parameters(), model2.named_parameters()):
        if p.requires_grad:
            assert torch.equal(p, q), n
    tr.train_step()
    tr2.train_step()
    assert torch.allclose(model.memory_attention.query[0].weight, model2.memory_attention.query[0].weight)
    loaded = load_adapter_checkpoint(SparseKVEagleDrafter(_cfg()), path)
    assert loaded["format"] == "sparsecache.sparse-kv-eagle-adapter.v2"


def test_evaluation_modes_and_disabled_memory_invariance():
    model, bank, cos, sin, tr = _trainer()
    rows = list(range(6))
    res = {m: evaluate_drafter(model, bank, rows, cos, sin, memory_mode=m, batch=4)
           for m in ("exact", "zero", "shuffled", "disabled")}
    for r in res.values():
        assert 0.0 <= r["mean_accepted_prefix"] <= 4 and 0.0 <= r["teacher_forced_top1"] <= 1.0
    a = evaluate_drafter(model, bank, rows, cos, sin, memory_mode="disabled")
    assert a == res["disabled"]


def test_batch_indices_are_disjoint_across_ranks():
    model, bank, cos, sin, tr = _trainer()
    tr.world, tr.local_batch = 2, 2
    tr.rank = 0
    a, _ = tr.batch_indices(0)
    tr.rank = 1
    b, _ = tr.batch_indices(0)
    assert not set(a) & set(b)


def _trainer_with(defer: bool):
    torch.manual_seed(0)
    cfg = _cfg()
    model = random_eagle_drafter(cfg, seed=0, std=0.2)
    model.bind_target_embedding(torch.randn(cfg.target_vocab_size, cfg.target_hidden_size))
    model.freeze_eagle()
    configure_trainable_modules(model, train_fc=False, train_midlayer=False, adapter_scale_init=0.0)
    bank = synthetic_bank(n_samples=8, horizon=5, n_layers=2, n_heads=2, n_seed=2, target_hidden=16, hidden=16,
                          vocab=24, visible=6, prompt_tokens=30, topk=4, device="cpu", head_dim=8)
    cos, sin = torch.randn(64, 8), torch.randn(64, 8)
    tcfg = DrafterTrainConfig(lr=3e-2, global_batch=4, use_graph=False, feature_weight=0.5,
                              defer_weight_grads=defer)
    return model, EagleDrafterTrainer(model, bank, cos, sin, tcfg)


def test_deferred_weight_gradients_equal_autograd():
    """One GEMM per adapter weight after the recurrence == autograd's per-position sums."""
    grads = {}
    for defer in (False, True):
        model, tr = _trainer_with(defer)
        assert (tr.stash is not None) == defer
        if defer:  # the four memory projections (2 layers x query/output) are deferred
            assert len(tr.stash.linears) == 4
        seen = []
        tr.opt.step = lambda tr=tr, seen=seen: seen.append(tr.flat.grad.clone())  # keep the gradient, no update
        tr.train_step()
        grads[defer] = seen[0]
        tr.release()
        assert all(type(m) is torch.nn.Linear for m in (*model.memory_attention.query, *model.memory_attention.output))
    a, b = grads[False], grads[True]
    assert float(a.abs().max()) > 0
    assert torch.allclose(a, b, rtol=1e-4, atol=1e-6), float((a - b).abs().max())


def test_flat_buckets_cover_the_buffer_once():
    _, tr = _trainer_with(True)
    late = [lin.weight for lin in tr.stash.linears]
    buckets = tr.flat.buckets(late)
    assert len(buckets) == 1 + len(late)
    cover = torch.zeros(tr.flat.padded, dtype=torch.int32)
    for ranges in buckets:
        for lo, hi in ranges:
            cover[lo:hi] += 1
    assert bool((cover == 1).all())
    for p, ranges in zip(late, buckets[1:]):
        (lo, hi), = ranges
        assert hi - lo == p.numel() and p.grad.data_ptr() == tr.flat.grad[lo:].data_ptr()


def test_weight_grad_stash_rejects_misuse():
    import pytest

    from sparsecache_b200.training.deferred_grad import WeightGradStash

    lin = torch.nn.Linear(8, 4, bias=False)
    st = WeightGradStash(torch.device("cpu"))
    st.register(lin)
    st.begin(rows_per_call=3, max_calls=2)
    assert st.xT[0].shape == (8, 64) and st.dyT[0].shape == (4, 64)  # padded to the GEMM's K tile
    st.next_call(0, lin.weight)
    st.next_call(0, lin.weight)
    with pytest.raises(RuntimeError):
        st.next_call(0, lin.weight)
    with pytest.raises(ValueError):
        st.put_x(0, 0, torch.zeros(5, 8))  # 5 rows where each call has 3
    with pytest.raises(ValueError):
        WeightGradStash(torch.device("cpu")).register(torch.nn.Linear(8, 4))  # biased linears are not deferred
