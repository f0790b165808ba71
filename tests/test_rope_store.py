"""RoPE relocation and the KV file format / dedup store (CPU)."""
import json
import math

import pytest
import torch

from sparsecache_b200.config import get_model_config
from sparsecache_b200.rope import (
    apply_rope,
    inverse_frequencies,
    relocate_key,
    relocate_positions,
    remove_rope,
    rope_cos_sin,
    rope_table,
)
from sparsecache_b200.store import (
    MANIFEST_FORMAT,
    DocumentKVStore,
    cache_bytes,
    compose_cache,
    config_fingerprint,
    load_cache,
    load_manifest,
    model_fingerprint,
    save_cache,
    slice_cache,
    stack_legacy,
)


def test_rope_round_trip():
    cfg = get_model_config("tiny")
    x = torch.randn(1, 2, 17, cfg.head_dim)
    cos, sin = rope_cos_sin(cfg, torch.arange(100, 117))
    y = apply_rope(x, cos, sin, sequence_dim=2)
    torch.testing.assert_close(remove_rope(y, cos, sin, sequence_dim=2), x, rtol=1e-5, atol=1e-5)


def test_relocation_equals_direct_rotation():
    cfg = get_model_config("llama3-8b")
    raw = torch.randn(1, 8, 40, 128)
    c0, s0 = rope_cos_sin(cfg, torch.arange(0, 40))
    c1, s1 = rope_cos_sin(cfg, torch.arange(1000, 1040))
    at_zero = apply_rope(raw, c0, s0, sequence_dim=2)
    moved = relocate_key(cfg, at_zero, source_start=0, target_start=1000)
    direct = apply_rope(raw, c1, s1, sequence_dim=2)
    torch.testing.assert_close(moved, direct, rtol=1e-4, atol=1e-4)
    assert relocate_key(cfg, at_zero, source_start=5, target_start=5) is at_zero


def test_llama3_scaling_bands():
    cfg = get_model_config("llama3-8b")
    inv = inverse_frequencies(cfg)
    base = 1.0 / (cfg.rope_theta ** (torch.arange(0, 128, 2).float() / 128))
    wavelen = 2 * math.pi / base
    # high frequencies unchanged, low frequencies divided by the factor
    assert torch.allclose(inv[wavelen < 8192 / 4], base[wavelen < 8192 / 4])
    assert torch.allclose(inv[wavelen > 8192], base[wavelen > 8192] / 8)
    tiny = get_model_config("tiny")
    assert torch.allclose(inverse_frequencies(tiny), 1.0 / (500000.0 ** (torch.arange(0, 64, 2).float() / 64)))


def test_rope_table_matches_cos_sin():
    cfg = get_model_config("tiny128")
    table = rope_table(cfg, 300)
    cos, sin = rope_cos_sin(cfg, torch.arange(300))
    assert torch.equal(table[:, 0::2], cos[:, :64])
    assert torch.equal(table[:, 1::2], sin[:, :64])


def _cache(layers, heads, tokens, dim, seed):
    g = torch.Generator().manual_seed(seed)
    return tuple(
        (torch.randn(1, heads, tokens, dim, generator=g).to(torch.bfloat16),
         torch.randn(1, heads, tokens, dim, generator=g).to(torch.bfloat16))
        for _ in range(layers)
    )


def test_save_load_slice(tmp_path):
    cache = _cache(3, 2, 9, 64, 0)
    nbytes = save_cache(tmp_path / "c.safetensors", cache)
    assert nbytes == cache_bytes(cache)
    loaded = load_cache(tmp_path / "c.safetensors", expected_layers=3)
    for (k, v), (lk, lv) in zip(cache, loaded):
        assert torch.equal(k, lk) and torch.equal(v, lv)
    with pytest.raises(ValueError):
        load_cache(tmp_path / "c.safetensors", expected_layers=4)
    part = slice_cache(cache, 2, 5)
    assert part[0][0].shape == (1, 2, 3, 64)
    assert not list(tmp_path.glob("*.tmp"))


def test_manifest_compose(tmp_path):
    cfg = get_model_config("tiny")
    system = _cache(cfg.n_layers, cfg.n_kv_heads, 5, cfg.head_dim, 1)
    chunks = [_cache(cfg.n_layers, cfg.n_kv_heads, n, cfg.head_dim, 10 + n) for n in (4, 6)]
    save_cache(tmp_path / "system.safetensors", system)
    manifest = {"format": MANIFEST_FORMAT, "model": {"layers": cfg.n_layers},
                "system": {"file": "system.safetensors", "tokens": 5}, "chunks": []}
    src = 5
    for i, c in enumerate(chunks):
        save_cache(tmp_path / f"chunk_{i:02d}.safetensors", c)
        manifest["chunks"].append({"chunk_id": f"c{i}", "title": "t", "file": f"chunk_{i:02d}.safetensors",
                                   "tokens": c[0][0].shape[2], "source_start": 5})
    (tmp_path / "manifest.json").write_text(json.dumps(manifest))
    m = load_manifest(tmp_path / "manifest.json")
    composed, meta = compose_cache(cfg, m)
    assert composed[0][0].shape[2] == 15
    assert meta["prefix_tokens"] == 15 and meta["relocated_tokens"] == 6  # first chunk lands at 5
    expect = relocate_key(cfg, chunks[1][0][0], source_start=5, target_start=9)
    assert torch.equal(composed[0][0][:, :, 9:], expect)
    bad = dict(manifest, format="other")
    (tmp_path / "bad.json").write_text(json.dumps(bad))
    with pytest.raises(ValueError):
        load_manifest(tmp_path / "bad.json")


def test_fingerprints(tmp_path):
    (tmp_path / "config.json").write_text("{}")
    a = model_fingerprint(tmp_path)
    (tmp_path / "model.safetensors.index.json").write_text("{\"w\": 1}")
    assert model_fingerprint(tmp_path) != a
    cfg = get_model_config("tiny")
    assert config_fingerprint(cfg, 0) != config_fingerprint(cfg, 1)


def test_document_store_dedup_and_persistence(tmp_path):
    cfg = get_model_config("tiny")
    calls = []

    def producer(tokens):
        calls.append(tokens)
        return stack_legacy(_cache(cfg.n_layers, cfg.n_kv_heads, len(tokens), cfg.head_dim, len(calls)))

    store = DocumentKVStore(cfg, tier="cpu")
    docs = [(5, 6, 7), (8, 9), (5, 6, 7), (10,)]
    stats = store.produce(producer, docs)
    assert stats["unique_documents"] == 3 and stats["producer_calls"] == 3
    assert len(calls) == 3 and (5, 6, 7) in store
    assert store[(8, 9)].kv.shape == (cfg.n_layers, 2, cfg.n_kv_heads, 2, cfg.head_dim)
    fp = config_fingerprint(cfg, 0)
    store.save(tmp_path / "store", fp)
    again = DocumentKVStore.load(tmp_path / "store", cfg, fp, tier="cpu")
    assert torch.equal(again[(5, 6, 7)].kv, store[(5, 6, 7)].kv)
    with pytest.raises(ValueError):
        DocumentKVStore.load(tmp_path / "store", cfg, "wrong", tier="cpu")
