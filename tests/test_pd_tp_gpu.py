"""Prefill group -> decode group KV push between tensor-parallel groups (TPn -> TPn).

Ranks [0, tp) prefill with the push fused into the TP QKV GEMM epilogue (rank
i stores its kv heads' rows into decode rank tp + i's slot); ranks [tp, 2 tp)
wait (bounded, on the device) for their partner's last layer and seed, then
run the TP greedy decode.  Checks:
  * every decode rank's pushed K/V equals its partner's own cache bit for bit;
  * the decode group's tokens equal the prefill group's own TP decode of the
    same prompt from its local cache;
  * no bounded wait timed out.
TP1 -> TP1 runs on 2 GPUs, TP2 -> TP2 on 4, TP4 -> TP4 on 8.
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


def _worker(rank, world, tp, port, out_dir):
    import torch.distributed as dist

    from sparsecache_b200.config import get_model_config
    from sparsecache_b200.parallel.pd_tp import TPPD
    from sparsecache_b200.synthetic import make_requests

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    result = {"rank": rank}
    dep = None
    try:
        cfg = get_model_config("llama3-8b").with_layers(3)
        req = make_requests("tiny_plumbing", cfg)[1]
        T, n_new = req.prompt_tokens, 10
        dep = TPPD(cfg, tp, capacity=2048, push=True, seed=5)
        dep.ch.epoch = 1
        ids = torch.tensor(req.prompt, dtype=torch.int32, device=dev)
        dist.barrier()
        if dep.role == "prefill":
            dep.prefill(ids, n_new)
            torch.cuda.synchronize()
            dist.send(dep.ch.slot.data[:, :, :, :T].contiguous(), dep.partner)
            # the prefill group's own decode from its local cache (same steps on every prefill rank)
            dep.tpe.decode(dep.ch.slot, n_new - 1)
            torch.cuda.synchronize()
            local = dep.tokens(n_new)
            dist.send(torch.tensor(local, dtype=torch.int64, device=dev), dep.partner)
        else:
            dep.wait(0, timeout_s=20.0)
            mine = torch.empty_like(dep.ch.slots[0].data[:, :, :, :T].contiguous())
            dist.recv(mine, dep.partner)
            torch.cuda.synchronize()
            result["kv_bitwise_equal"] = bool(torch.equal(dep.ch.slots[0].data[:, :, :, :T], mine))
            dep.decode(T, n_new)
            torch.cuda.synchronize()
            result["pushed_tokens"] = dep.tokens(n_new)
            ref = torch.empty(n_new, dtype=torch.int64, device=dev)
            dist.recv(ref, dep.partner)
            result["prefill_group_tokens"] = ref.tolist()
        dep.check()
        result["ok"] = True
    except Exception as exc:  # noqa: BLE001
        result["error"] = repr(exc)
    finally:
        try:
            if dep is not None:
                dep.close()
        finally:
            with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
                json.dump(result, f)
            dist.destroy_process_group()


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_tp_prefill_group_pushes_to_tp_decode_group(tmp_path, tp):
    world = 2 * tp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, tp, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [json.loads((tmp_path / f"r{r}.json").read_text()) for r in range(world)]
    for r in res:
        assert "error" not in r, r
    for r in res[tp:]:
        assert r["kv_bitwise_equal"], r
        assert r["pushed_tokens"] == r["prefill_group_tokens"], r
