"""Tensor-parallel prefill with fused AG->GEMM / GEMM->RS against the single-GPU engine (2 GPUs)."""
import json
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist

    from sparsecache_b200.config import get_model_config
    from sparsecache_b200.models.engine import B200Engine, EngineWeights
    from sparsecache_b200.models.llama import LlamaOracle
    from sparsecache_b200.parallel.tp import TPEngine, TPGroup
    from sparsecache_b200.synthetic import make_requests

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    result = {"rank": rank}
    try:
        cfg = get_model_config("tiny128")
        oracle = LlamaOracle.random_init(cfg, seed=11, std=0.05)
        full = EngineWeights.from_oracle(oracle, dev)
        group = TPGroup()
        tpe = TPEngine.from_full(cfg, full, group, max_rows=1024)
        req = make_requests("tiny_plumbing", cfg)[0]
        T = req.prompt_tokens
        ids = torch.tensor(req.prompt, dtype=torch.int32, device=dev)
        slot = tpe.new_slot(2 * 1024)
        x, rows, Tp = tpe.prefill(ids, slot)
        torch.cuda.synchronize()
        tpe.check_status()
        ref = B200Engine(cfg, full, dev, max_positions=8192)
        rslot = ref.new_slot(2048)
        h = ref.prefill(ids, rslot).float()
        hn = h * torch.rsqrt(h.square().mean(-1, keepdim=True) + cfg.rms_eps) * full.norm.float()
        lo, hi = rank * rows, min((rank + 1) * rows, T)
        err = float(((x[: hi - lo].float() - hn[lo:hi]).abs().max() / hn[lo:hi].abs().max()).item())
        hkv = cfg.n_kv_heads // world
        kv_err = 0.0
        for layer in range(cfg.n_layers):
            a = slot.k(layer)[:, :T].float()
            b = rslot.k(layer)[rank * hkv:(rank + 1) * hkv, :T].float()
            kv_err = max(kv_err, float(((a - b).abs().max() / b.abs().max()).item()))
        result.update(hidden_rel_err=err, kv_rel_err=kv_err, rows=rows, padded=Tp, canaries=group.check_canaries())
        # TP decode (fused all-reduce GEMVs) vs single-GPU greedy decode
        n_new = 8
        for use_graph in (False, True):
            x, rows, Tp = tpe.prefill(ids, slot)
            tpe.first_token(x, rows, T, max_new=n_new)
            tpe.decode(slot, n_new - 1, use_graph=use_graph)
            torch.cuda.synchronize()
            tpe.check_status()
            result[f"tp_tokens_graph{int(use_graph)}"] = tpe.engine.generated_tokens(n_new).tolist()
        ref.first_token(h.to(torch.bfloat16)[T - 1:T], position=T, max_new=n_new)
        ref.decode(rslot, n_new - 1, max_new=n_new)
        result["ref_tokens"] = ref.generated_tokens(n_new).tolist()
        dist.barrier()
        tpe.close()
        dist.barrier()
    except Exception as exc:  # noqa: BLE001
        result["error"] = repr(exc)
    finally:
        with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
            json.dump(result, f)
        dist.destroy_process_group()


def test_tp2_prefill_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        res = json.loads((tmp_path / f"r{r}.json").read_text())
        assert "error" not in res, res
        assert res["hidden_rel_err"] < 3e-2, res
        assert res["canaries"] == [], res
        assert res["kv_rel_err"] < 3e-2, res
        # graph replay and eager steps agree exactly; the first tokens match the
        # single-GPU engine (partial sums are added in a different order, so
        # only the leading tokens are required to agree on a random model)
        assert res["tp_tokens_graph0"] == res["tp_tokens_graph1"], res
        assert res["tp_tokens_graph0"][:3] == res["ref_tokens"][:3], res


def _spec_worker(rank, world, port, out_dir):
    """TP CacheBlend vs the single-GPU engine, verify == decode, drafter vs module, lossless speculation."""
    import torch.distributed as dist

    from sparsecache_b200.config import CacheBlendConfig, get_model_config
    from sparsecache_b200.models.engine import B200Engine, EngineWeights
    from sparsecache_b200.models.llama import LlamaOracle
    from sparsecache_b200.models.sparse_kv_draft import stage_features
    from sparsecache_b200.models.sparse_kv_eagle import SparseKVEagleConfig, SparseKVEagleDrafter
    from sparsecache_b200.parallel.serve_tp import TPRAGServer
    from sparsecache_b200.parallel.tp import TPEngine, TPGroup
    from sparsecache_b200.parallel.tp_draft import TPDraftWeights, TPEagleDrafter, speculative_generate
    from sparsecache_b200.rope import rope_cos_sin
    from sparsecache_b200.store import DocumentKVStore
    from sparsecache_b200.synthetic import make_requests

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    result = {"rank": rank}
    try:
        cfg = get_model_config("tiny128")
        oracle = LlamaOracle.random_init(cfg, seed=11, std=0.05)
        full = EngineWeights.from_oracle(oracle, dev)
        group = TPGroup()
        tpe = TPEngine.from_full(cfg, full, group, max_rows=2048 // world)
        # the TP layers run the row-tile GEMM at every row count; the single-GPU reference does
        # the same here so that one rank reproduces its partial sums bit for bit
        import sparsecache_b200.models.engine as engine_module

        engine_module.USE_WIDE_GEMM = False
        ref = B200Engine(cfg, full, dev, max_positions=8192)
        req = make_requests("tiny_plumbing", cfg)[0]
        T, n_new = req.prompt_tokens, 12
        blend = CacheBlendConfig(check_layer=1, recompute_ratio=0.15)
        server = TPRAGServer(tpe, capacity=4096, blend=blend, budget=512, recent=128)
        server.produce([req])
        meta = server.prefill_request(req, mode="cacheblend", max_new=n_new)
        act_tp = meta["active"].tolist()
        tp_first = int(tpe.engine.generated_tokens(1)[0])
        # ---- single-GPU CacheBlend on the same documents
        store = DocumentKVStore(cfg, device=dev)

        def enc(tokens):
            blk = ref.new_slot(len(tokens))
            ref.prefill(torch.tensor(list(tokens), dtype=torch.int32, device=dev), blk)
            return blk.data

        store.produce(enc, req.documents)
        rslot = ref.new_slot(4096)
        ids = torch.tensor(req.prompt, dtype=torch.int32, device=dev)
        ref.compose(rslot, [store[d].kv for d in req.documents], first_slot=len(req.prefix), layer_begin=1)
        h_a, A, rmeta = ref.cacheblend(ids, rslot, prefix_tokens=len(req.prefix), suffix_tokens=len(req.suffix),
                                       blend=blend)
        act_ref = rmeta["active"].tolist()
        ref.first_token(h_a[A - 1:A], position=T, max_new=n_new)
        ref.decode(rslot, n_new - 1, max_new=n_new)
        result.update(active_overlap=len(set(act_tp) & set(act_ref)) / len(act_ref), active_equal=act_tp == act_ref,
                      first_tp=tp_first, first_ref=int(ref.generated_tokens(1)[0]),
                      ref_tokens=ref.generated_tokens(n_new).tolist())
        # ---- greedy TP decode from the CacheBlend state, then lossless speculation from the same state
        greedy = server.decode(req, meta, max_new=n_new, speculative=False)["tokens"]
        result["tp_greedy"] = greedy
        server.prefill_request(req, mode="cacheblend", max_new=n_new)
        # greedy through the verifier (tensor-core skinny GEMMs, one row per step): the
        # reference of the speculative loop; the decode path (GEMV) may differ only at ties
        plain = speculative_generate(tpe, None, server.slot, prompt_tokens=T, max_new=n_new)["tokens"]
        # the two verify backends on the same state: residual rows after the seed layers agree
        feats = {}
        for backend in ("gemv", "skinny"):
            tpe.verify_backend = backend
            server.prefill_request(req, mode="cacheblend", max_new=n_new)
            rows_t = torch.tensor(plain[:5], dtype=torch.int32, device=dev)
            tpe.verify(server.slot, rows_t, T)
            feats[backend] = tpe.engine.ws.bufs["tp_feat"].view(len(tpe.seed_layers), 8, cfg.d_model)[:, :5].float()
            feats[backend] = feats[backend].clone()
        tpe.verify_backend = "skinny"
        ref_f = feats["gemv"]
        result["verify_backends_rel_err"] = float(((feats["skinny"] - ref_f).abs().max() / ref_f.abs().max()).item())

        class Oracle:  # proposes the verifier's greedy continuation with its last draft corrupted
            gamma = 4

            def propose(self, slot, first_token, seed_row, position, use_graph=True):
                k = position - T + 1  # index in ``plain`` of the token after first_token
                want = (plain[k:k + 4] + [0, 0, 0, 0])[:4]
                want[3] = (want[3] + 1) % cfg.vocab
                return torch.tensor(want, dtype=torch.int32, device=dev)

        server.prefill_request(req, mode="cacheblend", max_new=n_new)
        spec = speculative_generate(tpe, Oracle(), server.slot, prompt_tokens=T, max_new=n_new)
        result.update(oracle_equal=spec["tokens"] == plain, oracle_accepted=spec["accepted"])
        # ---- TP drafter vs the torch module (same weights, same target KV)
        dcfg = SparseKVEagleConfig(target_hidden_size=512, hidden_size=512, intermediate_size=1024, head_dim=128,
                                   num_attention_heads=4, num_key_value_heads=2, num_memory_heads=2,
                                   num_memory_layers=3, num_seed_layers=3, target_vocab_size=cfg.vocab,
                                   draft_vocab_size=1024)
        torch.manual_seed(5)
        module = SparseKVEagleDrafter(dcfg)
        with torch.no_grad():
            module.adapter_scale.fill_(0.0)
            module.memory_attention.layer_gates.copy_(torch.tensor([0.3, -0.2, 0.1]))
        module = module.to(device=dev, dtype=torch.bfloat16)
        module.stage_layer_bias.float()  # the stage scalars enter in fp32
        module.bind_target_embedding(full.embed)
        mem_layers = (0, 1, 2)
        drafter = TPEagleDrafter(tpe, dcfg, TPDraftWeights.from_module(module, rank, world, dev),
                                 memory_layers=mem_layers, gamma=2)
        server.drafter = drafter
        server.prefill_request(req, mode="cacheblend", max_new=n_new)
        view = server.memory_view(T, meta["active"])
        drafter.set_request(view, T, max_new=n_new)
        b = tpe.engine._decode_buffers()
        rows = torch.empty(1, dtype=torch.int32, device=dev)
        rows.copy_(b["log"][0:1])
        pred0 = tpe.verify(server.slot, rows, T)
        feat = tpe.engine.ws.bufs["tp_feat"].view(len(tpe.seed_layers), 8, cfg.d_model)
        seed = feat[:, 0].clone()
        drafts = drafter.propose(server.slot, pred0[0:1].clone(), seed, T + 1).tolist()
        hid_tp = drafter.hid.float().clone()
        # module with the target KV of the single-GPU engine (full heads), teacher-forced on the TP drafts
        full_view = torch.cat((view.long(), torch.tensor([T], device=dev)))
        mk = torch.stack([rslot.k(l)[:, full_view] for l in mem_layers])
        mv = torch.stack([rslot.v(l)[:, full_view] for l in mem_layers])
        # the TP slot holds the same composed prompt; re-run the verify row on the reference for position T
        ref_tok = torch.tensor([int(rows.item())], dtype=torch.int32, device=dev)
        ref.verify(rslot, ref_tok, position=T)
        mk[:, :, -1] = torch.stack([rslot.k(l)[:, T] for l in mem_layers])
        mv[:, :, -1] = torch.stack([rslot.v(l)[:, T] for l in mem_layers])
        cos, sin = rope_cos_sin(cfg, torch.arange(T + 1, T + 3), device=dev, dtype=torch.bfloat16)
        stage = stage_features(view.numel() / T, T, dtype=torch.bfloat16, device=dev)
        with torch.no_grad():
            state = module.init_state(seed.unsqueeze(0))
            tok = pred0[0:1].long().view(1, 1)
            ok = []
            for p in range(2):
                f, state = module.step(tok, state, cos[p:p + 1], sin[p:p + 1], mk, mv, stage)
                logits = module.lm_head(f).float().view(-1)
                d_id = int(module.target_to_draft[drafts[p]].item()) if drafts[p] < cfg.vocab else -1
                d_id = drafts[p] if d_id < 0 else d_id
                ok.append(bool(logits[d_id] >= logits.max() - 0.02 * logits.abs().max()))
                tok = torch.tensor([[drafts[p]]], device=dev)
            hid_ref = state[0].float().view(1, -1)
        result.update(draft_near_argmax=ok,
                      draft_hidden_rel_err=float(((hid_tp - hid_ref).abs().max() / hid_ref.abs().max()).item()))
        # lossless with the real drafter
        server.prefill_request(req, mode="cacheblend", max_new=n_new)
        out = server.decode(req, meta, max_new=n_new, speculative=True)
        result.update(drafter_equal=out["tokens"] == plain, drafter_accepted=out["accepted"])
        # batched decode of 3 sequences == each sequence through the verifier on its own
        reqs3 = make_requests("tiny_plumbing", cfg)[:3]
        server.produce(reqs3)
        bslots = tpe.batch_slots(3, 4096)
        own_slot, firsts, alone = server.slot, [], []
        for r3, sl in zip(reqs3, bslots):
            server.slot = sl
            server.prefill_request(r3, mode="cacheblend", max_new=n_new)
            firsts.append(int(tpe.engine.generated_tokens(1)[0]))
            alone.append(speculative_generate(tpe, None, sl, prompt_tokens=r3.prompt_tokens, max_new=n_new)["tokens"])
        server.slot = own_slot
        for use_graph in (False, True):
            tpe.start_batch(bslots, firsts, [r3.prompt_tokens for r3 in reqs3], max_new=n_new)
            tpe.decode_batch(bslots, n_new - 1, use_graph=use_graph)
            result[f"batch_equal_graph{int(use_graph)}"] = tpe.batch_tokens(3, n_new) == alone
        tpe.check_status()
        torch.cuda.synchronize()
        result["canaries"] = group.check_canaries()
        tpe.engine.release_graphs()
        drafter._graph = None
        dist.barrier()
        tpe.close()
        dist.barrier()
    except Exception as exc:  # noqa: BLE001
        import traceback

        result["error"] = repr(exc) + traceback.format_exc()[-2000:]
    finally:
        with open(os.path.join(out_dir, f"s{rank}.json"), "w") as f:
            json.dump(result, f)
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2])
def test_tp_cacheblend_and_speculative_decoding(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_spec_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        res = json.loads((tmp_path / f"s{r}.json").read_text())
        assert "error" not in res, res.get("error")
        # one rank: the same partial sums as the single-GPU engine -> identical selection
        if world == 1:
            assert res["active_equal"], res
        assert res["active_overlap"] > 0.97, res
        assert res["first_tp"] == res["first_ref"], res
        assert res["tp_greedy"][:3] == res["ref_tokens"][:3], res
        assert res["verify_backends_rel_err"] < 3e-2, res
        assert res["oracle_equal"] and max(res["oracle_accepted"]) == 3, res
        assert all(res["draft_near_argmax"]), res
        assert res["draft_hidden_rel_err"] < 5e-2, res
        assert res["drafter_equal"], res
        assert res["batch_equal_graph0"] and res["batch_equal_graph1"], res
        assert res["canaries"] == [], res
