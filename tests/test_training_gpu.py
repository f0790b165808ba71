"""GPU tests of the drafter-training kernels: K13 memory attention (forward
and dq) and the fused AdamW against plain PyTorch fp32 references, the
graph-captured trainer against its eager form, and the peer-memory data
parallel optimizer against the single-GPU step (2 GPUs)."""
import json
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _memory_batch(dev, S=3, L=2, T=300, H=4, D=128, seed=0):
    from sparsecache_b200.ops.sparse_attention import MemoryBatch

    g = torch.Generator(device="cpu").manual_seed(seed)
    keys = torch.randn(S, L, T, H, D, generator=g).to(dev, torch.bfloat16)
    values = torch.randn(S, L, T, H, D, generator=g).to(dev, torch.bfloat16)
    n_vis = torch.tensor([T, 37, 181], dtype=torch.int32)[:S]
    idx = torch.zeros(S, T, dtype=torch.int32)
    for s in range(S):
        sel = torch.randperm(T, generator=g)[: int(n_vis[s])].sort().values
        idx[s, : sel.numel()] = sel.to(torch.int32)
    return MemoryBatch(keys, values, idx.to(dev), n_vis.to(dev), None)


def test_memory_attention_forward_and_dq_match_fp32_reference(cuda_device):
    dev = cuda_device
    mem = _memory_batch(dev)
    rows = torch.tensor([2, 0, 1, 1, 2], dtype=torch.int32, device=dev)
    mem = mem.with_rows(rows)
    for t in (1, 3):
        q = (torch.randn(5, 4, t, 128, device=dev) * 0.5).to(torch.bfloat16).requires_grad_(True)
        for layer in range(2):
            out = mem.attend(layer, q)
            qr = q.detach().float().requires_grad_(True)
            ref = mem.attend_reference(layer, qr)  # fp32 math on the same bf16 memory
            assert (out.float() - ref).abs().max().item() < 2e-2
            g = torch.randn_like(ref)
            (out.float() * g).sum().backward()
            (ref * g).sum().backward()
            err = (q.grad.float() - qr.grad).abs().max().item()
            scale = qr.grad.abs().max().item()
            assert err < 2e-2 * max(1.0, scale), (t, layer, err, scale)
            q.grad = None


def test_memory_attention_heads_major_matches_sdpa(cuda_device):
    from sparsecache_b200.models.sparse_kv_draft import _memory_attention_reference, sparse_memory_attention

    dev = cuda_device
    q = torch.randn(2, 8, 5, 128, device=dev).to(torch.bfloat16)
    k = torch.randn(8, 211, 128, device=dev).to(torch.bfloat16)
    v = torch.randn(8, 211, 128, device=dev).to(torch.bfloat16)
    out = sparse_memory_attention(q, k, v)
    ref = _memory_attention_reference(q.float(), k.float(), v.float())
    assert (out.float() - ref).abs().max().item() < 2e-2


def test_fused_adamw_matches_torch_adamw_with_clipping(cuda_device):
    from sparsecache_b200.training.drafter_trainer import DrafterTrainConfig, FlatTrainables, FusedAdamW

    dev = cuda_device
    torch.manual_seed(0)
    a = torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.Linear(96, 33)).to(dev)
    b = torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.Linear(96, 33)).to(dev)
    b.load_state_dict(a.state_dict())
    flat = FlatTrainables(list(a.parameters()))
    opt = FusedAdamW(flat, DrafterTrainConfig(lr=3e-3, weight_decay=0.05, grad_clip=0.5))
    ref = torch.optim.AdamW(b.parameters(), lr=3e-3, weight_decay=0.05)
    x = torch.randn(16, 64, device=dev)
    for _ in range(4):
        flat.grad.zero_()
        a(x).square().sum().backward()
        opt.step()
        ref.zero_grad()
        b(x).square().sum().backward()
        torch.nn.utils.clip_grad_norm_(b.parameters(), 0.5)
        ref.step()
    for p, q in zip(a.parameters(), b.parameters()):
        assert torch.allclose(p, q, atol=2e-6, rtol=1e-5)
    assert float(opt.state[0]) == 4.0


def test_frozen_tc_linear_forward_and_input_grad(cuda_device):
    """Frozen projection on the tcgen05 GEMM: Y = X W^T and dX = dY W against fp32."""
    from sparsecache_b200.ops.linear import use_tc_for_frozen_linears

    dev = cuda_device
    lin = torch.nn.Linear(512, 768, bias=False).to(dev, torch.bfloat16)
    lin.weight.requires_grad_(False)
    assert use_tc_for_frozen_linears(torch.nn.Sequential(lin)) == ["0"]
    x = torch.randn(3, 37, 512, device=dev).to(torch.bfloat16).requires_grad_(True)
    y = lin(x)
    g = torch.randn_like(y)
    (y.float() * g.float()).sum().backward()
    w = lin.weight.float()
    ref = x.detach().float() @ w.T
    assert y.shape == (3, 37, 768) and y.dtype == torch.bfloat16
    assert ((y.float() - ref).abs().max() / ref.abs().max()).item() < 1e-2
    dref = g.float() @ w
    assert ((x.grad.float() - dref).abs().max() / dref.abs().max()).item() < 1e-2


@pytest.mark.parametrize("G,P", [(4, 1), (4, 97), (8, 256), (1, 33)])
def test_recurrent_attention_forward_backward_match_fp32(cuda_device, G, P):
    """K14: one new position over P past keys (GQA group G), forward and q / k / v gradients
    against fp32 SDPA on repeated K/V."""
    from sparsecache_b200.ops.linear import recurrent_attention

    dev = cuda_device
    B, hkv = 3, 2
    g = torch.Generator(device="cpu").manual_seed(G * 1000 + P)
    q = torch.randn(B, hkv * G, 1, 128, generator=g).to(dev, torch.bfloat16).requires_grad_(True)
    k = torch.randn(B, hkv, P, 128, generator=g).to(dev, torch.bfloat16).requires_grad_(True)
    v = torch.randn(B, hkv, P, 128, generator=g).to(dev, torch.bfloat16).requires_grad_(True)
    out = recurrent_attention(q, k, v)
    dout = torch.randn(out.shape, generator=g).to(dev, torch.bfloat16)
    (out.float() * dout.float()).sum().backward()
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(qr, kr.repeat_interleave(G, 1), vr.repeat_interleave(G, 1))
    (ref * dout.float()).sum().backward()
    for name, a, b in (("out", out, ref), ("dq", q.grad, qr.grad), ("dk", k.grad, kr.grad), ("dv", v.grad, vr.grad)):
        # a single key makes the softmax constant: dq is 0 up to rounding, so errors are taken
        # relative to at least 1e-2
        err = ((a.float() - b).abs().max() / b.abs().max().clamp_min(1e-2)).item()
        assert err < 2e-2, (name, err)


def test_trainer_with_tc_linears_matches_library_linears(cuda_device):
    """The trainer with the frozen trunk on the tcgen05 GEMM tracks the one on autograd's linears
    (bf16 rounding of the projections only)."""
    dev = cuda_device
    m1, t1 = _small_setup(dev, use_graph=True, tc_linears=True)
    m2, t2 = _small_setup(dev, use_graph=True, tc_linears=False)
    assert t1.tc_linears and not t2.tc_linears
    t1.warmup_and_capture(warmup=2)
    t2.warmup_and_capture(warmup=2)
    for _ in range(3):
        t1.train_step()
        t2.train_step()
        torch.cuda.synchronize()
        a, b = float(t1.loss), float(t2.loss)
        assert abs(a - b) <= 2e-2 * max(1.0, abs(b)), (a, b)
    w1 = m1.memory_attention.query[0].weight
    w2 = m2.memory_attention.query[0].weight
    assert (w1 - w2).abs().max().item() < 5e-3
    t1.release()
    t2.release()


def _small_setup(dev, seed=0, global_batch=4, use_graph=True, distributed=False, tc_linears=False, defer=True):
    from sparsecache_b200.models.sparse_kv_eagle import SparseKVEagleConfig
    from sparsecache_b200.training.drafter_trainer import (DrafterTrainConfig, EagleDrafterTrainer,
                                                           prepare_for_training, random_eagle_drafter)
    from sparsecache_b200.training.teacher import synthetic_bank

    cfg = SparseKVEagleConfig(target_hidden_size=256, hidden_size=256, intermediate_size=512, head_dim=128,
                              num_attention_heads=2, num_key_value_heads=1, num_memory_heads=2,
                              num_memory_layers=3, num_seed_layers=3, target_vocab_size=1024,
                              draft_vocab_size=512)
    model = random_eagle_drafter(cfg, seed=seed, std=0.05)
    model.freeze_eagle()
    model.adapter_scale.data.fill_(0.0)
    prepare_for_training(model, dev)
    g = torch.Generator().manual_seed(5)
    model.bind_target_embedding((torch.randn(1024, 256, generator=g) * 0.5).to(dev, torch.bfloat16))
    bank = synthetic_bank(n_samples=8, horizon=12, n_layers=3, n_heads=2, n_seed=3, target_hidden=256, hidden=256,
                          vocab=512, visible=96, prompt_tokens=500, topk=8, device=dev, seed=3)
    pos = torch.arange(1024, dtype=torch.float32)[:, None] * torch.logspace(0, -4, 64)[None, :]
    cos = torch.cat((pos.cos(), pos.cos()), -1)
    sin = torch.cat((pos.sin(), pos.sin()), -1)
    tcfg = DrafterTrainConfig(lr=1e-3, global_batch=global_batch, use_graph=use_graph, tc_linears=tc_linears,
                              defer_weight_grads=defer)
    return model, EagleDrafterTrainer(model, bank, cos, sin, tcfg, distributed=distributed)


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (1024, 4096, 2048), (4096, 1024, 200)])
def test_gemm_f32_matches_fp32_matmul(cuda_device, M, N, K):
    """Tensor-core GEMM with an fp32 result (the deferred weight gradients) vs an fp32 matmul."""
    from sparsecache_b200 import ops

    g = torch.Generator(device=cuda_device).manual_seed(M + N + K)
    a = torch.randn(M, K, device=cuda_device, generator=g).to(torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, generator=g).to(torch.bfloat16)
    out = torch.full((M, N), float("nan"), device=cuda_device)
    ops.ext().gemm_f32(a, w, out)
    ref = a.float() @ w.float().t()
    err = ((out - ref).abs().max() / ref.abs().max()).item()
    assert err < 1e-5, err


def test_deferred_weight_gradients_match_autograd(cuda_device):
    """Adapter weight gradients from one GEMM per weight after the recurrence vs autograd's per-position
    products (bf16 sums over positions there, fp32 here)."""
    grads = {}
    for defer in (False, True):
        model, tr = _small_setup(cuda_device, use_graph=False, defer=defer)
        assert (tr.stash is not None) == defer
        seen = []
        tr.opt.step = lambda tr=tr, seen=seen: seen.append(tr.flat.grad.clone())
        tr.train_step()
        torch.cuda.synchronize()
        grads[defer] = seen[0]
        tr.release()
    a, b = grads[False], grads[True]
    rel = ((a - b).norm() / a.norm()).item()
    assert a.norm().item() > 0 and rel < 1e-2, rel


def test_graph_captured_trainer_matches_eager(cuda_device):
    dev = cuda_device
    m1, t1 = _small_setup(dev, use_graph=True)
    m2, t2 = _small_setup(dev, use_graph=False)
    t1.warmup_and_capture(warmup=3)
    t2.warmup_and_capture(warmup=3)
    losses = []
    for _ in range(4):
        t1.train_step()
        t2.train_step()
        losses.append((float(t1.loss), float(t2.loss)))
    torch.cuda.synchronize()
    assert all(abs(a - b) <= 1e-3 * max(1.0, abs(b)) for a, b in losses), losses
    w1 = m1.memory_attention.query[0].weight
    w2 = m2.memory_attention.query[0].weight
    assert torch.allclose(w1, w2, atol=1e-4), (w1 - w2).abs().max()
    assert t1.steps_done == t2.steps_done == 7
    t1.release()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    res = {"rank": rank}
    try:
        model, tr = _small_setup(dev, global_batch=4, use_graph=True, distributed=True)
        tr.warmup_and_capture(warmup=2)
        for _ in range(3):
            tr.train_step()
        torch.cuda.synchronize()
        tr.opt.check()
        res["weight"] = model.memory_attention.query[1].weight.float().cpu().flatten()[:4096].tolist()
        res["steps"] = tr.steps_done
        dist.barrier()
        tr.release()
        # one eager step from a fresh start: the first moment of this rank's optimizer shard is
        # (1 - beta1) * clip * (rank-averaged gradient), linear in the gradient
        model2, tr2 = _small_setup(dev, global_batch=4, use_graph=False, distributed=True)
        tr2.train_step()
        torch.cuda.synchronize()
        tr2.opt.check()
        torch.save({"exp_avg": tr2.opt.exp_avg.cpu(), "numel": tr2.flat.numel, "shard": tr2.flat.shard(world)},
                   os.path.join(out_dir, f"m1_rank{rank}.pt"))
        dist.barrier()
        tr2.release()
    except Exception as exc:  # noqa: BLE001
        res["error"] = repr(exc)
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(res, f)
        dist.destroy_process_group()


def test_data_parallel_optimizer_matches_single_gpu(tmp_path, cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_dp_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(2)]
    for r in res:
        assert "error" not in r, r.get("error")
    assert res[0]["weight"] == res[1]["weight"]  # replicas identical bit for bit
    model, tr = _small_setup(cuda_device, global_batch=4, use_graph=False)
    init = model.memory_attention.query[1].weight.float().cpu().flatten()[:4096].clone()
    tr.warmup_and_capture(warmup=2)
    for _ in range(3):
        tr.train_step()
    ref = model.memory_attention.query[1].weight.float().cpu().flatten()[:4096]
    got = torch.tensor(res[0]["weight"])
    # Adam normalises every element's step, so bf16 rounding differences between one 4-row and two
    # 2-row batches flip the sign of near-zero updates: after five steps compare only the direction
    d_ref, d_got = ref - init, got - init
    assert torch.nn.functional.cosine_similarity(d_got, d_ref, dim=0).item() > 0.9
    # the exact check: after one step from the same start, the concatenated first-moment shards of
    # the two ranks equal the single-GPU first moment (the gradient of the 4-row batch, averaged)
    m1 = [torch.load(tmp_path / f"m1_rank{r}.pt") for r in range(2)]
    m_dp = torch.cat([m["exp_avg"] for m in m1])[: m1[0]["numel"]]
    model3, tr3 = _small_setup(cuda_device, global_batch=4, use_graph=False)
    tr3.train_step()
    torch.cuda.synchronize()
    m_ref = tr3.opt.exp_avg[: tr3.flat.numel].cpu()
    rel = ((m_dp - m_ref).norm() / m_ref.norm()).item()
    assert rel < 2e-2, rel

