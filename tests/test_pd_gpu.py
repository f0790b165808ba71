"""Prefill -> decode KV push over NVLink peer memory (2 GPUs).

Rank 0 prefills with the push fused into its QKV GEMM epilogue: every layer's
rotated K/V rows are stored into rank 1's serving slot and the layer's flag is
released.  Rank 1 waits (bounded, on the device) for the last layer and the
seed token, then decodes greedily.  Checks:
  * the pushed K/V on rank 1 equal rank 0's own cache bit for bit;
  * rank 1's tokens equal a single-GPU prefill + greedy decode on rank 1;
  * a bounded wait on a flag that nothing sets records a time-out status and
    returns, and the context stays usable afterwards.
"""
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
    from sparsecache_b200.models.engine import B200Engine
    from sparsecache_b200.parallel.pd import PDChannel, decode_request, prefill_request
    from sparsecache_b200.synthetic import make_requests

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    result = {"rank": rank}
    ch = None
    try:
        cfg = get_model_config("llama3-8b").with_layers(3)
        engine = B200Engine.random(cfg, seed=3, device=dev, max_positions=16384)
        req = make_requests("tiny_plumbing", cfg)[0]
        T, n_new = req.prompt_tokens, 12
        ids = torch.tensor(req.prompt, dtype=torch.int32, device=dev)
        role = "prefill" if rank == 0 else "decode"
        ch = PDChannel(engine, role=role, capacity=2048, prefill_rank=0, decode_rank=1)
        ch.epoch = 1
        dist.barrier()
        if role == "prefill":
            prefill_request(ch, ids, n_new)
            torch.cuda.synchronize()
            # the prefill side's own cache, for the bitwise comparison
            dist.send(ch.slot.data[:, :, :, :T].contiguous(), 1)
        else:
            decode_request(ch, T, n_new, timeout_s=20.0)
            torch.cuda.synchronize()
            result["status_after_push"] = int(ch.status.item())
            pushed_tokens = engine.generated_tokens(n_new).tolist()
            mine = torch.empty_like(ch.slot.data[:, :, :, :T].contiguous())
            dist.recv(mine, 0)
            result["kv_bitwise_equal"] = bool(torch.equal(ch.slot.data[:, :, :, :T], mine))
            # single-GPU reference on this GPU: local prefill + greedy decode
            ref_slot = engine.new_slot(2048)
            h = engine.prefill(ids, ref_slot)
            engine.first_token(h[T - 1:T], position=T, max_new=n_new)
            engine.decode(ref_slot, n_new - 1, max_new=n_new)
            result["pushed_tokens"] = pushed_tokens
            result["local_tokens"] = engine.generated_tokens(n_new).tolist()
            # a flag nothing sets: the bounded wait times out into the status word
            ext = engine.ext
            ext.wait_flag(ch.flags, cfg.n_layers - 1, ch.epoch + 100, int(0.5e9), ch.status)
            torch.cuda.synchronize()
            result["status_after_timeout"] = int(ch.status.item())
            ch.status.zero_()
            probe = torch.arange(4, device=dev, dtype=torch.float32).sum()
            result["context_usable"] = float(probe.item()) == 6.0
        dist.barrier()
    except Exception as exc:  # noqa: BLE001
        result["error"] = repr(exc)
    finally:
        try:
            if ch is not None:
                dist.barrier()
                ch.close()
        finally:
            with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
                json.dump(result, f)
            dist.destroy_process_group()


def test_pd_push_matches_local_prefill(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    res = [json.loads((tmp_path / f"r{r}.json").read_text()) for r in range(2)]
    for r in res:
        assert "error" not in r, r
    dec = res[1]
    assert dec["status_after_push"] == 0
    assert dec["kv_bitwise_equal"]
    assert dec["pushed_tokens"] == dec["local_tokens"]
    assert dec["status_after_timeout"] == 6  # kStatusTimeoutPeerFlag
    assert dec["context_usable"]
