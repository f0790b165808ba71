"""CacheBlend algorithm on the CPU plumbing decoder (2 layers, d 256, fp32)."""
import math

import pytest
import torch

from sparsecache_b200.cacheblend import (
    cacheblend_prefill_oracle,
    compose_documents,
    deviation_scores,
    recompute_count,
    select_active,
    selection_checksum,
)
from sparsecache_b200.config import CacheBlendConfig, get_model_config
from sparsecache_b200.models.llama import LlamaOracle
from sparsecache_b200.synthetic import make_requests, workload_summary


@pytest.fixture(scope="module")
def tiny():
    cfg = get_model_config("tiny")
    model = LlamaOracle.random_init(cfg, seed=0)
    reqs = make_requests("tiny_plumbing", cfg)
    return cfg, model, reqs


def _composed(cfg, model, req):
    docs = [model.encode_local(d) for d in req.documents]
    return compose_documents(cfg, docs, prefix_tokens=len(req.prefix))


def test_workloads():
    cfg = get_model_config("tiny")
    s = workload_summary(make_requests("tiny_plumbing", cfg))
    assert s["requests"] == 8 and s["document_uses"] == 80
    assert s["repeated_uses"] == 16  # 20% of 80 slots
    big = workload_summary(make_requests("llama8b_rag", get_model_config("llama3-8b")))
    assert big["document_uses"] == 1500 and big["unique_documents"] == 1255 and big["repeated_uses"] == 245
    r = make_requests("llama8b_rag", get_model_config("llama3-8b"))[0]
    assert len(r.prefix) == 32 and 12 <= len(r.suffix) <= 40
    assert all(40 <= len(d) <= 400 for d in r.documents)
    assert max(max(r.prompt) for r in make_requests("llama8b_rag", get_model_config("llama3-8b"))) < 128000


def test_ratio_one_reproduces_full_prefill(tiny):
    cfg, model, reqs = tiny
    for req in reqs[:3]:
        full_logits, full_cache = model.prefill(req.prompt)
        out = cacheblend_prefill_oracle(model, req.prompt, _composed(cfg, model, req),
                                        prefix_tokens=len(req.prefix), suffix_tokens=len(req.suffix),
                                        blend=CacheBlendConfig(recompute_ratio=1.0))
        assert torch.equal(out.logits, full_logits)
        for (k, v), (fk, fv) in zip(out.cache, full_cache):
            assert torch.equal(k, fk) and torch.equal(v, fv)
        eos = set(cfg.eos_token_ids)
        T = len(req.prompt)
        assert model.greedy(out.logits, out.cache, T, 24, eos) == model.greedy(full_logits, full_cache, T, 24, eos)


@pytest.mark.parametrize("metric", ["value", "key", "kv", "value_l1"])
@pytest.mark.parametrize("keep_prefix", [True, False])
def test_selection_contract(tiny, metric, keep_prefix):
    cfg, model, reqs = tiny
    req = reqs[1]
    blend = CacheBlendConfig(recompute_ratio=0.15, deviation_metric=metric, keep_prefix=keep_prefix)
    out = cacheblend_prefill_oracle(model, req.prompt, _composed(cfg, model, req),
                                    prefix_tokens=len(req.prefix), suffix_tokens=len(req.suffix), blend=blend)
    n_doc = req.document_tokens
    k = max(1, math.ceil(0.15 * n_doc))
    assert out.selected_positions.numel() == k
    active = out.active_positions.tolist()
    assert active == sorted(active)
    T = len(req.prompt)
    assert set(range(T - len(req.suffix), T)) <= set(active)
    prefix = set(range(len(req.prefix)))
    assert (prefix <= set(active)) == keep_prefix
    assert out.metadata["document_tokens_selected"] == k
    assert out.metadata["selection_checksum"] == selection_checksum(out.selected_positions)


def test_deviation_and_select_helpers():
    fk = torch.zeros(1, 2, 5, 4)
    ck = torch.zeros(1, 2, 5, 4)
    fv = torch.zeros(1, 2, 5, 4)
    cv = torch.zeros(1, 2, 5, 4)
    fv[:, :, 3] = 2.0
    fk[:, :, 1] = 1.0
    assert int(deviation_scores(fk, fv, ck, cv, "value").argmax()) == 3
    assert int(deviation_scores(fk, fv, ck, cv, "key").argmax()) == 1
    assert deviation_scores(fk, fv, ck, cv, "kv_l1")[3] == 16.0
    scores = torch.tensor([0.1, 0.9, 0.5, 0.2])
    active, sel = select_active(scores, doc_begin=2, doc_end=6, total=8, ratio=0.5, keep_prefix=True)
    assert active.tolist() == [0, 1, 3, 4, 6, 7]
    assert recompute_count(0, 0.5) == 0 and recompute_count(10, 0.01) == 1
    with pytest.raises(ValueError):
        CacheBlendConfig(recompute_ratio=0.0)
    with pytest.raises(ValueError):
        CacheBlendConfig(deviation_metric="cosine")
    assert CacheBlendConfig(deviation_metric="kv_l1").dev_mode == 7


def test_gradual_filtering_schedule(tiny):
    """Several check layers with non-increasing ratios (relative to the original document count)."""
    cfg, model, reqs = tiny
    req = reqs[2]
    comp = _composed(cfg, model, req)
    kw = dict(prefix_tokens=len(req.prefix), suffix_tokens=len(req.suffix))
    full_logits, _ = model.prefill(req.prompt)
    ones = cacheblend_prefill_oracle(model, req.prompt, comp, **kw,
                                     blend=CacheBlendConfig(check_layers=(0, 1), recompute_ratios=(1.0, 1.0)))
    assert torch.equal(ones.logits, full_logits)
    first = cacheblend_prefill_oracle(model, req.prompt, comp, **kw,
                                      blend=CacheBlendConfig(check_layer=0, recompute_ratio=0.5))
    grad = cacheblend_prefill_oracle(model, req.prompt, comp, **kw,
                                     blend=CacheBlendConfig(check_layers=(0, 1), recompute_ratios=(0.5, 0.15)))
    n_doc = req.document_tokens
    assert grad.selected_positions.numel() == recompute_count(n_doc, 0.15)
    assert set(grad.selected_positions.tolist()) <= set(first.selected_positions.tolist())
    assert grad.metadata["layer_document_trace"] == [1.0, 0.5]
    assert grad.metadata["check_layers"] == [0, 1] and grad.metadata["recompute_ratios"] == [0.5, 0.15]
    with pytest.raises(ValueError, match="misses the target"):
        CacheBlendConfig(check_layers=(0, 1), recompute_ratios=(0.5, 0.15),
                         target_average_recompute_ratio=0.5).check_target(2)
    with pytest.raises(ValueError):
        CacheBlendConfig(check_layers=(1, 0), recompute_ratios=(0.3, 0.2))
    with pytest.raises(ValueError):
        CacheBlendConfig(check_layers=(0, 1), recompute_ratios=(0.2, 0.3))
    # the reference runner's example: 15% true layer-average over 32 layers
    ex = CacheBlendConfig(check_layers=(0, 1, 2), recompute_ratios=(0.30, 0.20, 0.11379310344827587),
                          target_average_recompute_ratio=0.15)
    assert abs(ex.check_target(32) - 0.15) < 1e-9
    assert abs(CacheBlendConfig().check_target(32) - 0.203125) < 1e-12


def test_runner_flags_build_the_schedule():
    import argparse

    from sparsecache_b200.pipelines.reuse import blend_config_from_args

    base = dict(deviation_metric="kv_l1", max_new_tokens=16, check_layer=1, recompute_ratio=0.15,
                blend_check_layers=None, recompute_ratios=None, target_average_recompute_ratio=None)
    b = blend_config_from_args(argparse.Namespace(**base))
    assert b.schedule == ((1, 0.15),) and b.deviation_metric == "kv_l1" and b.dev_mode == 1 | 2 | 4
    g = blend_config_from_args(argparse.Namespace(**{**base, "blend_check_layers": "0,1,2",
                                                     "recompute_ratios": "0.30,0.20,0.11379310344827587",
                                                     "target_average_recompute_ratio": 0.15}))
    assert g.schedule[0] == (0, 0.30) and abs(g.check_target(32) - 0.15) < 1e-9
    with pytest.raises(SystemExit):
        blend_config_from_args(argparse.Namespace(**{**base, "blend_check_layers": "0,1"}))
