"""Hugging Face Llama / Mistral checkpoint directories load into the oracle (and so the engine) with the
same logits as the transformers model: HF config mapping (GQA, head_dim, rope_theta, llama3 rope scaling,
EOS ids), sharded safetensors through the index, tied embeddings."""
import pytest
import torch

transformers = pytest.importorskip("transformers")


def _check(model, tmp_path, *, shard="100KB"):
    from sparsecache_b200.models.checkpoint import load_config, load_oracle

    model.save_pretrained(tmp_path, max_shard_size=shard, safe_serialization=True)
    assert (tmp_path / "model.safetensors.index.json").exists()  # sharded
    oracle = load_oracle(tmp_path)
    ids = torch.randint(3, model.config.vocab_size, (1, 150), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        want = model(ids).logits[0, -1].float()
    got, _ = oracle.prefill(ids[0].tolist())
    assert torch.allclose(got.float(), want, atol=2e-4, rtol=2e-4), (got - want).abs().max()
    return load_config(tmp_path)


def test_llama_with_llama3_rope_scaling(tmp_path):
    cfg = transformers.LlamaConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                                   rope_theta=500000.0, eos_token_id=[7, 9], bos_token_id=1,
                                   rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                                 "high_freq_factor": 4.0, "original_max_position_embeddings": 64})
    torch.manual_seed(0)
    mc = _check(transformers.LlamaForCausalLM(cfg).eval(), tmp_path)
    assert (mc.n_kv_heads, mc.head_dim, mc.eos_token_ids) == (2, 32, (7, 9))
    assert mc.rope_scaling is not None and mc.rope_scaling.original_max_position_embeddings == 64


def test_mistral_with_tied_embeddings(tmp_path):
    cfg = transformers.MistralConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                     num_attention_heads=4, num_key_value_heads=1, rope_theta=1e6,
                                     sliding_window=None, tie_word_embeddings=True)
    torch.manual_seed(1)
    mc = _check(transformers.MistralForCausalLM(cfg).eval(), tmp_path)
    assert mc.n_kv_heads == 1 and mc.rope_theta == 1e6


def test_unsupported_families_are_refused():
    from sparsecache_b200.models.checkpoint import config_from_hf

    base = {"num_hidden_layers": 2, "hidden_size": 64, "num_attention_heads": 4, "intermediate_size": 128,
            "vocab_size": 100}
    with pytest.raises(ValueError, match="architecture"):
        config_from_hf({**base, "architectures": ["Qwen3ForCausalLM"]})
    with pytest.raises(ValueError, match="sliding"):
        config_from_hf({**base, "sliding_window": 16, "max_position_embeddings": 4096})
    with pytest.raises(ValueError, match="rope scaling"):
        config_from_hf({**base, "rope_scaling": {"rope_type": "yarn", "factor": 4.0}})


@pytest.mark.parametrize("tp", [1, 2])
def test_tensor_parallel_shards_read_from_the_checkpoint(tmp_path, tp):
    """Each rank's shard read with safetensors slices equals slicing the full engine weights."""
    from sparsecache_b200.models.checkpoint import checkpoint_shard, load_oracle
    from sparsecache_b200.models.engine import EngineWeights
    from sparsecache_b200.parallel.tp import shard_weights

    cfg = transformers.LlamaConfig(vocab_size=256, hidden_size=128, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, tie_word_embeddings=True)
    torch.manual_seed(2)
    transformers.LlamaForCausalLM(cfg).save_pretrained(tmp_path, max_shard_size="100KB")
    full = EngineWeights.from_oracle(load_oracle(tmp_path), "cpu")
    for rank in range(tp):
        mc, got = checkpoint_shard(tmp_path, rank, tp)
        want = shard_weights(full, mc, rank, tp)
        assert torch.equal(got.embed, want.embed) and torch.equal(got.lm_head, want.lm_head)
        for a, b in zip(got.layers, want.layers):
            for name in ("ln1", "w_qkv", "w_o", "ln2", "w_gu", "w_down"):
                assert torch.equal(getattr(a, name), getattr(b, name)), name


def test_shard_and_config_errors(tmp_path):
    from sparsecache_b200.models.checkpoint import checkpoint_shard, save_checkpoint
    from sparsecache_b200.config import get_model_config
    from sparsecache_b200.models.llama import LlamaOracle

    save_checkpoint(tmp_path, LlamaOracle.random_init(get_model_config("tiny"), seed=0))
    with pytest.raises(ValueError, match="divide"):
        checkpoint_shard(tmp_path, 0, 3)  # 4 heads / 2 kv heads do not split three ways
    with pytest.raises(ValueError, match="divide"):
        checkpoint_shard(tmp_path, 0, 2)  # FFN 688 is not a whole number of 128-row gate/up blocks per rank
