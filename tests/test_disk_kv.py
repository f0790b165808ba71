"""Layer-wise disk KV streaming (native loader, host mode on CPU; device mode on a B200)."""
import pytest
import torch

from sparsecache_b200 import ops
from sparsecache_b200.config import get_model_config
from sparsecache_b200.serving.disk_kv import DiskKVStore, LayerwiseDiskKV, safetensors_extents
from sparsecache_b200.store import load_cache

needs_ext = pytest.mark.skipif(not ops.available(), reason="extension not built")


def _blocks(cfg, lengths, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(cfg.n_layers, 2, cfg.n_kv_heads, n, cfg.head_dim, generator=g).to(torch.bfloat16)
            for n in lengths]


def test_chunk_kv_files_and_header_extents(tmp_path):
    cfg = get_model_config("tiny")
    store = DiskKVStore(tmp_path, cfg)
    (blk,) = _blocks(cfg, [37])
    p = store.put((5, 6, 7), blk)
    assert (5, 6, 7) in store and store.put((5, 6, 7), blk) == p
    legacy = load_cache(p, expected_layers=cfg.n_layers)
    assert torch.equal(legacy[1][0][0], blk[1, 0]) and legacy[1][0].shape == (1, cfg.n_kv_heads, 37, cfg.head_dim)
    ext = safetensors_extents(p)
    raw = p.read_bytes()
    off, nb, shape, dtype = ext["layer_001.value"]
    assert dtype == "BF16" and shape == (1, cfg.n_kv_heads, 37, cfg.head_dim)
    got = torch.frombuffer(bytearray(raw[off:off + nb]), dtype=torch.bfloat16).view(shape[1:])
    assert torch.equal(got, blk[1, 1])


@needs_ext
@pytest.mark.parametrize("n_buffers,n_threads", [(1, 1), (2, 4)])
def test_native_loader_host_mode_streams_layers(tmp_path, n_buffers, n_threads):
    cfg = get_model_config("tiny")
    store = DiskKVStore(tmp_path, cfg)
    lengths = [19, 64, 7, 33]
    blocks = _blocks(cfg, lengths, seed=3)
    paths = [store.put((i, n), b) for i, (n, b) in enumerate(zip(lengths, blocks))]
    loader = LayerwiseDiskKV(cfg, "cpu", host=True, staging_bytes=1 << 12, n_buffers=n_buffers,
                             n_threads=n_threads)
    layers = list(range(1, cfg.n_layers))
    for _ in range(2):  # a second request reuses the loader and its buffers
        out = loader.start(paths, layers)
        for l in layers:
            loader.wait_layer(l)
            for b, o in zip(blocks, out):
                assert torch.equal(o[l], b[l])
        stats = loader.join()
        assert stats["layers"] == len(layers) and stats["layers_enqueued"] == len(layers)
        assert stats["bytes"] == sum(b[1:].numel() * 2 for b in blocks)
    assert loader.staging_bytes >= max(sum(b[0].numel() * 2 for b in blocks), 1 << 12)


@needs_ext
def test_native_loader_reports_missing_file(tmp_path):
    cfg = get_model_config("tiny")
    loader = LayerwiseDiskKV(cfg, "cpu", host=True)
    with pytest.raises(Exception):
        loader.start([tmp_path / "absent.safetensors"], [0])


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["async", "sync"])
def test_cacheblend_from_disk_matches_hbm(tmp_path, cuda_device, mode):
    from sparsecache_b200.config import CacheBlendConfig
    from sparsecache_b200.models.engine import B200Engine
    from sparsecache_b200.serving.disk_kv import blend_from_disk
    from sparsecache_b200.serving.server import RAGServer
    from sparsecache_b200.store import DocumentKVStore
    from sparsecache_b200.synthetic import make_requests

    cfg = get_model_config("tiny128")
    eng = B200Engine.random(cfg, seed=2, device=cuda_device, max_positions=8192)
    blend = CacheBlendConfig(check_layer=1, recompute_ratio=0.15)
    store = DocumentKVStore(cfg, device=cuda_device)
    server = RAGServer(eng, store, capacity=4096, blend=blend)
    reqs = make_requests("tiny_plumbing", cfg)[:2]
    server.produce(reqs)
    disk = DiskKVStore(tmp_path, cfg)
    disk.put_all(store)
    loader = LayerwiseDiskKV(cfg, cuda_device)
    for r in reqs:
        ids = torch.tensor(r.prompt, dtype=torch.int32, device=cuda_device)
        slot = eng.new_slot(4096)
        eng.compose(slot, [store[d].kv for d in r.documents], first_slot=len(r.prefix), layer_begin=1)
        h_ref, A, meta_ref = eng.cacheblend(ids, slot, prefix_tokens=len(r.prefix), suffix_tokens=len(r.suffix),
                                            blend=blend)
        h_ref, act_ref = h_ref.clone(), meta_ref["active"].clone()
        kv_ref = slot.data[:, :, :, :r.prompt_tokens].clone()
        slot2 = eng.new_slot(4096)
        (h, A2, meta), _ = blend_from_disk(eng, slot2, r, ids, disk, loader, blend=blend, mode=mode)
        stats = loader.join()
        torch.cuda.synchronize()
        assert A2 == A and torch.equal(meta["active"], act_ref)
        assert torch.equal(h, h_ref)
        assert torch.equal(slot2.data[:, :, :, :r.prompt_tokens], kv_ref)
        assert stats["layers"] == cfg.n_layers - 1
