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
    from sparsecache_b200.pipelines.reuse import (EngineStageModel, evaluate_request, prepare_request,
                                                  run_progressive_cacheblend)
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
    blocks = [server.store[d].kv for d in prep.request.documents]
    model = EngineStageModel(server, prep, document_blocks=blocks)
    assert model.final_decode([], 12) == list(one_shot.token_ids)
    res = run_progressive_cacheblend(server, prep, blocks, draft_tokens=4, max_new_tokens=12)
    assert len(res["tokens"]) == 12 and res["repairs"] >= 2
    row = evaluate_request(server, prep, max_new_tokens=12, draft_tokens=4)
    assert set(row["arms"]) == {"full", "cacheblend", "progressive"}
    assert row["arms"]["cacheblend"]["tokens"] == list(one_shot.token_ids)


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
