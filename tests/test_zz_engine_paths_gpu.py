"""GPU comparisons of two engine paths against the fp32 PyTorch oracle: CacheBlend with gradual
filtering (several check layers) and the drafter-teacher extraction (prefill hooks, CUDA-graph greedy
decode, continuation prefill).  The file sorts after the other GPU suites, so a run that stops at the
first failure has already run them."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel_max(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


def test_gradual_cacheblend_engine_matches_oracle(cuda_device):
    """Check layers 1 and 2 of the 3-layer geometry at ratios 0.5 then 0.2 of the documents: the engine keeps
    the oracle's rows (near-ties in the bf16 deviation ranking may swap a few) and its last-row logits agree."""
    from sparsecache_b200.cacheblend import cacheblend_prefill_oracle, compose_documents
    from sparsecache_b200.config import CacheBlendConfig, get_model_config
    from sparsecache_b200.models.engine import B200Engine
    from sparsecache_b200.models.llama import LlamaOracle
    from sparsecache_b200.serving.server import RAGServer
    from sparsecache_b200.store import DocumentKVStore
    from sparsecache_b200.synthetic import make_requests

    cfg = get_model_config("tiny128")
    oracle = LlamaOracle.random_init(cfg, seed=0, std=0.05)
    engine = B200Engine.from_oracle(oracle, cuda_device, max_positions=8192)
    store = DocumentKVStore(cfg, tier="hbm", device=cuda_device)
    req = make_requests("tiny_plumbing", cfg)[1]
    blend = CacheBlendConfig(check_layers=(1, 2), recompute_ratios=(0.5, 0.2), max_new_tokens=12)
    RAGServer(engine, store, capacity=4096, blend=blend).produce([req])
    composed = compose_documents(cfg, [oracle.encode_local(d) for d in req.documents], prefix_tokens=len(req.prefix))
    ref = cacheblend_prefill_oracle(oracle, req.prompt, composed, prefix_tokens=len(req.prefix),
                                    suffix_tokens=len(req.suffix), blend=blend)
    ids = torch.tensor(req.prompt, dtype=torch.int32, device=cuda_device)
    slot = engine.new_slot(2048)
    engine.compose(slot, [store[d].kv for d in req.documents], first_slot=len(req.prefix), layer_begin=1)
    h_a, A, meta = engine.cacheblend(ids, slot, prefix_tokens=len(req.prefix), suffix_tokens=len(req.suffix),
                                     blend=blend)
    torch.cuda.synchronize()
    assert A == ref.active_positions.numel() and meta["check_layers"] == [1, 2]
    got = set(meta["active"][:A].cpu().tolist())
    want = set(ref.active_positions.tolist())
    assert len(got & want) / len(want) > 0.85
    logits = oracle.lm_head(oracle.norm(h_a[A - 1:A].float().cpu()))[0]
    assert _rel_max(logits, ref.logits) < 0.1


def test_engine_teacher_extraction_matches_oracle(cuda_device):
    """Teacher fields of the B200 engine (prefill hooks, graph decode, continuation prefill) against the
    plain-PyTorch oracle run along the engine's own continuation tokens."""
    from sparsecache_b200.config import get_model_config
    from sparsecache_b200.models.engine import B200Engine
    from sparsecache_b200.models.llama import LlamaOracle
    from sparsecache_b200.training.teacher import extract_teacher, extract_teacher_oracle

    def rel(a, b):
        return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-6))

    cfg = get_model_config("tiny128")
    oracle = LlamaOracle.random_init(cfg, seed=3, std=0.05, dtype=torch.bfloat16)
    engine = B200Engine.from_oracle(oracle, device=cuda_device)
    prompt = torch.randint(4, cfg.vocab, (300,), generator=torch.Generator().manual_seed(1), dtype=torch.int32)
    kw = dict(kv_layers=(0, 2), seed_layers=(1, 2), continuation_tokens=6, teacher_topk=16, page_size=64)
    eng = extract_teacher(engine, [prompt], keep_full_memory=True, **kw)[0].tensors
    ref = extract_teacher_oracle(oracle.float(), [prompt], continuation_ids=[eng["input_ids"]], **kw)[0].tensors
    assert set(eng) == set(ref)
    for name in ("memory_keys", "memory_values", "seed_hidden", "teacher_hidden", "continuation_seed_hidden"):
        assert eng[name].shape == ref[name].shape, name
        assert rel(eng[name], ref[name]) < 3e-2, name
    assert (eng["priority_page_scores"] - ref["priority_page_scores"]).abs().max() < 2e-2
    assert (eng["teacher_topk_logprobs"][:, 0] - ref["teacher_topk_logprobs"][:, 0]).abs().max() < 5e-2
    assert torch.allclose(eng["query_cos"].float(), ref["query_cos"].float(), atol=1e-2)
    assert torch.equal(eng["prompt_ids"], ref["prompt_ids"])
    # greedy agreement wherever the oracle's top-2 margin is clear of bf16 noise
    margin = ref["teacher_topk_logprobs"][:, 0] - ref["teacher_topk_logprobs"][:, 1]
    clear = margin > 0.1
    assert torch.equal(eng["labels"][clear], ref["labels"][clear])
