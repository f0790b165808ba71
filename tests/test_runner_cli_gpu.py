"""Command-line runners on the GPU, at tiny geometry: the reuse pipeline reading its model from a
model directory, and the producer-side proposal benchmark (dense seed vs seed + drafter proposal).
Their host parts are tested on the CPU; these runs check that the runners drive the engine end to
end and write the rows their aggregators read."""
import json

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_reuse_pipeline_from_model_directory(tmp_path, cuda_device):
    from sparsecache_b200.models.checkpoint import random_checkpoint
    from sparsecache_b200.pipelines.reuse import main

    model_dir = random_checkpoint(tmp_path / "model", "tiny128", seed=3, std=0.05)
    out = tmp_path / "rows.jsonl"
    main(["--model-dir", str(model_dir), "--workload", "tiny_plumbing", "--requests", "2", "--warmup", "1",
          "--max-new-tokens", "8", "--draft-tokens", "4", "--store-tier", "pinned", "--output", str(out)])
    lines = [json.loads(x) for x in out.read_text().splitlines()]
    assert lines[0]["protocol"]["model"] == str(model_dir)
    rows = lines[1:]
    assert len(rows) == 2
    for row in rows:
        arms = row["arms"]
        assert "progressive" in arms and len(arms) >= 2
        for arm in arms.values():
            assert len(arm["tokens"]) == 8 and arm["ttft_ms"] > 0


def test_producer_side_proposal_benchmark(tmp_path, cuda_device):
    from sparsecache_b200.models.sparse_kv_eagle import SparseKVEagleConfig
    from sparsecache_b200.pipelines.pd_source import main

    dcfg = SparseKVEagleConfig(target_hidden_size=512, hidden_size=512, intermediate_size=1024, head_dim=128,
                               num_attention_heads=4, num_key_value_heads=2, num_memory_heads=2,
                               num_memory_layers=3, num_seed_layers=3, target_vocab_size=4096,
                               draft_vocab_size=1024)
    cfg_path = tmp_path / "drafter.json"
    cfg_path.write_text(json.dumps(dcfg.to_dict()))
    out_dir = tmp_path / "source"
    out = main(["--model", "tiny128", "--workload", "tiny_plumbing", "--requests", "2", "--warmup", "1",
                "--horizon", "3", "--memory-layers", "0,1,2", "--seed-layers", "0,1,2",
                "--drafter-config", str(cfg_path), "--bootstrap-samples", "50", "--output-dir", str(out_dir)])
    assert out["samples"] == 2
    assert out["seed_match_fraction"] == 1.0  # both arms run the same prefill
    for p in out["paired"]:
        assert len(p["proposal_token_ids"]) == 3 and p["eagle_proposal_ready_ms"] > 0
    summary = json.loads((out_dir / "summary.json").read_text())
    assert set(summary["bandwidths"]) == {"25", "50", "100"}
    torch.cuda.synchronize()
