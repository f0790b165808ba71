"""Paged decode attention, batched verification and the progressive chain on the GPU."""
import math

import pytest
import torch

from sparsecache_b200.config import get_model_config
from sparsecache_b200.models.llama import LlamaOracle
from sparsecache_b200.serving.progressive import (
    Document,
    TrancheStager,
    continuous_graft_chain,
    stage_document_sets,
)
from sparsecache_b200.synthetic import make_requests

pytestmark = pytest.mark.gpu


def test_paged_decode_attention(cuda_device):
    from sparsecache_b200 import ops

    ext = ops.ext()
    H, Hkv, cap, M = 8, 2, 1500, 3
    kc = torch.randn(Hkv, cap, 128, device=cuda_device).to(torch.bfloat16)
    vc = torch.randn(Hkv, cap, 128, device=cuda_device).to(torch.bfloat16)
    q = torch.randn(M, H * 128, device=cuda_device).to(torch.bfloat16)
    n_prompt = 901
    perm = torch.randperm(1200)[:n_prompt]
    tail = torch.arange(1300, 1300 + M)
    view = torch.cat([perm, tail]).to(torch.int32).to(cuda_device)
    nv = torch.tensor([n_prompt + M], dtype=torch.int32, device=cuda_device)
    pos = torch.tensor([0], dtype=torch.int32, device=cuda_device)
    out = torch.empty(M, H * 128, device=cuda_device, dtype=torch.bfloat16)
    for splits in (8, 16):
        ext.attention_decode(q, kc, vc, pos, H, 1 / math.sqrt(128), splits, out, page_table=view, page_shift=0,
                             n_virtual=nv)
        torch.cuda.synchronize()
        keys = view.long()
        G = H // Hkv
        qh = q.float().view(M, H, 128).transpose(0, 1)
        k = kc[:, keys].float().repeat_interleave(G, 0)
        v = vc[:, keys].float().repeat_interleave(G, 0)
        s = qh @ k.transpose(1, 2) / math.sqrt(128)
        vis = torch.arange(keys.numel(), device=cuda_device)[None, :] <= (n_prompt + torch.arange(M, device=cuda_device))[:, None]
        s = s.masked_fill(~vis[None], float("-inf"))
        ref = (torch.softmax(s, -1) @ v).transpose(0, 1).reshape(M, -1)
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.fixture(scope="module")
def engine_setup():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from sparsecache_b200.models.engine import B200Engine

    cfg = get_model_config("tiny128")
    oracle = LlamaOracle.random_init(cfg, seed=7, std=0.05)
    return cfg, B200Engine.from_oracle(oracle, "cuda:0", max_positions=8192)


def test_batched_verify_matches_sequential_decode(engine_setup):
    cfg, engine = engine_setup
    req = make_requests("tiny_plumbing", cfg)[2]
    T = req.prompt_tokens
    slot = engine.new_slot(T + 64)
    h = engine.prefill(torch.tensor(req.prompt, dtype=torch.int32, device=engine.device), slot)
    engine.first_token(h[T - 1:T], position=T, max_new=8)
    engine.decode(slot, 7, max_new=8, use_graph=False)
    toks = engine.generated_tokens(8).tolist()
    preds = engine.verify(slot, torch.tensor(toks[:7], dtype=torch.int32), position=T).tolist()
    assert preds == toks[1:8]


def test_continuous_chain_is_exact(engine_setup):
    cfg, engine = engine_setup
    dev = engine.device
    req = make_requests("tiny_plumbing", cfg)[1]
    T, P, S = req.prompt_tokens, len(req.prefix), len(req.suffix)
    # producer side: full prompt KV and the seed token
    slot_p = engine.new_slot(T + 64)
    h = engine.prefill(torch.tensor(req.prompt, dtype=torch.int32, device=dev), slot_p)
    engine.first_token(h[T - 1:T], position=T, max_new=16)
    seed = int(engine.generated_tokens(1).item())
    source = slot_p.data[:, :, :, :T].cpu().pin_memory()
    docs = [Document(d, start=b, end=e) for d, (b, e) in zip(req.documents, req.document_ranges())]
    ranking = [4, 0, 9, 2, 7, 1, 8, 3, 6, 5]
    stages = stage_document_sets(ranking, docs, (0.1, 0.4, 0.7, 1.0))
    slot_d = engine.new_slot(T + 64)
    stager = TrancheStager(source, slot_d, prefix_tokens=P, documents=docs, suffix_tokens=S, ranking=ranking,
                           selected_sets=stages, transport_gbps=0.5, device=dev)
    stager.pack()
    res = continuous_graft_chain(engine, stager, seed_token=seed, prompt_tokens=T, max_draft_tokens=4,
                                 max_new_tokens=12)
    assert res.verifier_calls == 1 and len(res.draft_tokens) >= 1
    assert 0 <= res.accepted <= len(res.draft_tokens)
    # full-target baseline on the same compact cache: seed, then plain greedy decode
    slot_f = engine.new_slot(T + 64)
    slot_f.data[:, :, :, :T].copy_(torch.cat(stager._packed, dim=3).to(dev))
    b = engine._decode_buffers(16)
    b["ids"][:1].fill_(seed)
    engine.ext.embedding(b["ids"][:1], engine.w.embed, b["h"][:1])
    b["gen"].zero_()
    engine.set_decode_state(position=T)
    engine.decode(slot_f, 11, max_new=16, use_graph=False)
    full = [seed] + engine.generated_tokens(11).tolist()
    assert list(res.token_ids) == full


def test_fixed_view_control_is_exact_and_traced(engine_setup):
    """The fixed first-stage control drafts on the anchor view only; output stays exact."""
    cfg, engine = engine_setup
    dev = engine.device
    req = make_requests("tiny_plumbing", cfg)[1]
    T, P, S = req.prompt_tokens, len(req.prefix), len(req.suffix)
    slot_p = engine.new_slot(T + 64)
    h = engine.prefill(torch.tensor(req.prompt, dtype=torch.int32, device=dev), slot_p)
    engine.first_token(h[T - 1:T], position=T, max_new=16)
    seed = int(engine.generated_tokens(1).item())
    source = slot_p.data[:, :, :, :T].cpu().pin_memory()
    docs = [Document(d, start=b, end=e) for d, (b, e) in zip(req.documents, req.document_ranges())]
    ranking = list(range(len(docs)))
    stages = stage_document_sets(ranking, docs, (0.2, 0.6, 1.0))
    outs = []
    for grow in (True, False):
        stager = TrancheStager(source, engine.new_slot(T + 64), prefix_tokens=P, documents=docs, suffix_tokens=S,
                               ranking=ranking, selected_sets=stages, transport_gbps=0.5, device=dev)
        stager.pack()
        res = continuous_graft_chain(engine, stager, seed_token=seed, prompt_tokens=T, max_draft_tokens=4,
                                     max_new_tokens=12, grow_view=grow)
        rec = res.pipeline_record()
        assert rec["trace"][-1]["verified"] and rec["trace"][-1]["accepted_pending"] == res.accepted
        assert sum(t["drafted"] for t in rec["trace"]) == len(res.draft_tokens)
        if not grow:
            assert all(t["stage"] == 0 for t in rec["trace"][:-1])
        outs.append(list(res.token_ids))
    assert outs[0] == outs[1]  # both verified on the full KV: identical greedy output
