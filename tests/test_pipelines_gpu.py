"""Progressive CacheBlend reuse pipeline on the engine (tiny head_dim-128 geometry):
the final stage's repaired model decodes exactly what one-shot CacheBlend
serves, and the progressive chain (commit window 1) produces the full horizon."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_progressive_cacheblend_final_stage_matches_one_shot(cuda_device):
    from sparsecache_b200.config import CacheBlendConfig, get_model_config
    from sparsecache_b200.models.engine import B200Engine
    from sparsecache_b200.models.llama import LlamaOracle
    from sparsecache_b200.pipelines.reuse import (EngineStageModel, evaluate_request, host_blocks,
                                                  prepare_request, run_progressive_cacheblend)
    from sparsecache_b200.serving.doc_stager import PinnedDocumentStager
    from sparsecache_b200.serving.server import RAGServer
    from sparsecache_b200.store import DocumentKVStore
    from sparsecache_b200.synthetic import make_requests

    cfg = get_model_config("tiny128")
    engine = B200Engine.from_oracle(LlamaOracle.random_init(cfg, seed=5, std=0.05), cuda_device, max_positions=8192)
    reqs = make_requests("tiny_plumbing", cfg)[:2]
    server = RAGServer(engine, DocumentKVStore(cfg, tier="hbm", device=cuda_device), capacity=4096,
                       blend=CacheBlendConfig(check_layer=1, recompute_ratio=0.15, max_new_tokens=12))
    server.produce(reqs)
    prep = prepare_request(reqs[0], schedule="sequential", fractions=(0.3, 0.6, 1.0))
    one_shot = server.serve(prep.request, mode="cacheblend", max_new_tokens=12, sync=True)
    blocks = host_blocks(server, prep.request)
    assert all(b.is_pinned() for b in blocks)
    stager = PinnedDocumentStager(blocks, prep.selected_sets, device=cuda_device, layer_begin=1)
    model = EngineStageModel(server, prep, stager=stager)
    assert model.final_decode([], 12) == list(one_shot.token_ids)
    moved = stager.finish()
    assert moved["launched_stages"] == 3
    assert moved["total_bytes"] == sum(b[1:].numel() * 2 for b in blocks)
    res = run_progressive_cacheblend(server, prep, blocks, draft_tokens=4, max_new_tokens=12)
    assert len(res["tokens"]) == 12 and res["repairs"] >= 2
    ser = run_progressive_cacheblend(server, prep, blocks, draft_tokens=4, max_new_tokens=12, overlap=False)
    assert ser["tokens"] == res["tokens"] and ser["transfer"]["total_bytes"] == res["transfer"]["total_bytes"]
    pinned = DocumentKVStore(cfg, tier="pinned")
    for d in prep.request.documents:
        if d not in pinned:
            pinned.put(d, server.store[d].kv)
    row = evaluate_request(server, prep, max_new_tokens=12, draft_tokens=4, pinned_store=pinned)
    assert set(row["arms"]) == {"full", "cacheblend", "progressive"}
    assert row["arms"]["cacheblend"]["tokens"] == list(one_shot.token_ids)
    prog = row["arms"]["progressive"]
    assert prog["serial_pipeline_token_match"] and prog["serial_response_ms"] > 0
    assert prog["transfer"]["first_stage_h2d_ms"] > 0


def test_stage_prompt_holds_only_arrived_documents(cuda_device):
    """An early stage repairs prefix + arrived documents + suffix, the suffix at
    its final positions: with ratio 1.0 its first token equals the fp32 oracle's
    full prefill of that stage prompt with the same positions."""
    from sparsecache_b200.config import CacheBlendConfig, get_model_config
    from sparsecache_b200.models.engine import B200Engine
    from sparsecache_b200.models.llama import LlamaOracle
    from sparsecache_b200.pipelines.reuse import EngineStageModel, host_blocks, prepare_request
    from sparsecache_b200.serving.doc_stager import PinnedDocumentStager
    from sparsecache_b200.serving.server import RAGServer
    from sparsecache_b200.store import DocumentKVStore
    from sparsecache_b200.synthetic import make_requests

    cfg = get_model_config("tiny128")
    oracle = LlamaOracle.random_init(cfg, seed=9, std=0.05)
    engine = B200Engine.from_oracle(oracle, cuda_device, max_positions=8192)
    req = make_requests("tiny_plumbing", cfg)[0]
    server = RAGServer(engine, DocumentKVStore(cfg, tier="hbm", device=cuda_device), capacity=4096,
                       blend=CacheBlendConfig(check_layer=1, recompute_ratio=1.0, max_new_tokens=4))
    server.produce([req])
    prep = prepare_request(req, schedule="sequential", fractions=(0.3, 1.0))
    stager = PinnedDocumentStager(host_blocks(server, prep.request), prep.selected_sets, device=cuda_device,
                                  layer_begin=1)
    model = EngineStageModel(server, prep, stager=stager)
    first = model.verify(0, [])[0]
    ids, gpos, _ = model._stage_prompt(0)
    with torch.no_grad():
        hidden, _ = oracle.forward_tokens(ids.long().cpu(), gpos.long().cpu())
        logits = oracle.logits(hidden[:, -1])[0]
    top2 = torch.topk(logits.float(), 2).values
    if float(top2[0] - top2[1]) > 0.05:  # a clear winner must agree
        assert first == int(logits.argmax())
    assert len(ids) < prep.request.prompt_tokens and int(gpos[-1]) == prep.request.prompt_tokens - 1
    stager.finish()


def test_draft_screens(cuda_device):
    from sparsecache_b200.config import get_model_config
    from sparsecache_b200.models.engine import B200Engine
    from sparsecache_b200.models.llama import LlamaOracle
    from sparsecache_b200.pipelines.screens import layer_draft_screen, sparse_page_crossover

    cfg = get_model_config("tiny128")
    engine = B200Engine.from_oracle(LlamaOracle.random_init(cfg, seed=6, std=0.05), cuda_device, max_positions=8192)
    prompt = list(range(5, 700))
    rows = layer_draft_screen(engine, prompt, {"all": list(range(cfg.n_layers)), "first_1": [0]}, draft_tokens=6)
    by = {r["pattern"]: r for r in rows}
    assert by["all"]["accepted_prefix"] == 5  # the full layer set drafts exactly the target's tokens
    assert 0 <= by["first_1"]["accepted_prefix"] <= 5 and by["first_1"]["ms_per_token"] > 0
    cross = sparse_page_crossover(engine, [2048], [0.1, 1.0], reps=3)
    assert len(cross) == 2 and all(c["draft_step_ms"] > 0 for c in cross)
    assert cross[1]["visible_fraction"] == 1.0
