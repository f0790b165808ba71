"""Public generation API on the B200 engine (tiny head_dim-128 geometry)."""
import pytest
import torch

from sparsecache_b200.config import get_model_config
from sparsecache_b200.modeling import baseline_generate, cacheblend_generate, direct_reuse_generate
from sparsecache_b200.models.llama import LlamaOracle
from sparsecache_b200.synthetic import make_requests

pytestmark = pytest.mark.gpu


def test_public_api_engine(cuda_device):
    from sparsecache_b200.models.engine import B200Engine

    cfg = get_model_config("tiny128")
    oracle = LlamaOracle.random_init(cfg, seed=3, std=0.05)
    engine = B200Engine.from_oracle(oracle, cuda_device, max_positions=8192)
    req = make_requests("tiny_plumbing", cfg)[0]
    full = req.prompt
    P = len(full) - len(req.suffix)
    base = baseline_generate(engine, full_ids=full, max_new_tokens=8, eos_token_ids=set())
    # prefix cache produced by the engine itself (exact full-prompt KV)
    slot = engine.new_slot(2048)
    engine.prefill(torch.tensor(full[:P], dtype=torch.int32, device=cuda_device), slot)
    cache = tuple((slot.data[i, 0, :, :P].unsqueeze(0).cpu(), slot.data[i, 1, :, :P].unsqueeze(0).cpu())
                  for i in range(cfg.n_layers))
    direct = direct_reuse_generate(engine, prefix_cache=cache, suffix_ids=req.suffix, max_new_tokens=8,
                                   eos_token_ids=set())
    assert direct.token_ids == base.token_ids
    blend = cacheblend_generate(engine, full_ids=full, prefix_cache=cache, system_tokens=len(req.prefix),
                                suffix_tokens=len(req.suffix), check_layer=1, recompute_ratio=1.0,
                                max_new_tokens=8, eos_token_ids=set(), deviation_metric="value", keep_prefix=True)
    assert blend.token_ids == base.token_ids
    part = cacheblend_generate(engine, full_ids=full, prefix_cache=cache, system_tokens=len(req.prefix),
                               suffix_tokens=len(req.suffix), check_layer=1, recompute_ratio=0.15,
                               max_new_tokens=8, eos_token_ids=set())
    assert part.metadata["document_tokens_selected"] == max(1, -(-(P - len(req.prefix)) * 15 // 100))
    assert base.prefill_ms > 0 and base.decode_ms > 0
