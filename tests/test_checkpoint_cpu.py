"""Base-model checkpoints (swarmlora_b200.checkpoint) on the CPU against
checkpoints written by transformers itself (LlamaForCausalLM.save_pretrained,
the format the reference's aggregator loads with from_pretrained): a
sharded one with an untied LM head and a single-file one with tied
embeddings load tensor for tensor, the config maps onto ModelConfig the way
the reference reads it, and broken checkpoints are refused."""
import json

import pytest
import torch

from swarmlora_b200 import checkpoint as ck

BF = torch.bfloat16


def _tiny(tie, scratch, name, shard):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=64, intermediate_size=96, num_attention_heads=2, num_key_value_heads=1,
                      head_dim=32, num_hidden_layers=2, vocab_size=128, rms_norm_eps=1e-5, rope_theta=500000.0,
                      tie_word_embeddings=tie, max_position_embeddings=131072,
                      rope_scaling={"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                    "original_max_position_embeddings": 8192, "rope_type": "llama3"})
    torch.manual_seed(3)
    model = LlamaForCausalLM(cfg).to(BF)
    with torch.no_grad():
        for p in model.parameters():
            p.copy_(torch.randn(p.shape) * 0.05)
    d = scratch / name
    model.save_pretrained(str(d), safe_serialization=True, max_shard_size=shard)
    return model, d


@pytest.mark.parametrize("tie,shard", [(False, "20KB"), (True, "10GB")])
def test_loads_what_transformers_writes(scratch, tie, shard):
    model, d = _tiny(tie, scratch, f"ckpt_{tie}", shard)
    assert (d / "model.safetensors.index.json").exists() == (not tie)
    base, cfg = ck.load_base(str(d), "cpu")
    assert (cfg.hidden, cfg.inter, cfg.layers, cfg.hq, cfg.hkv, cfg.head_dim, cfg.vocab) == (64, 96, 2, 2, 1, 32, 128)
    assert cfg.eps == 1e-5 and cfg.rope_theta == 500000.0 and cfg.rope_scaling["rope_type"] == "llama3"
    sd = model.state_dict()
    for l in range(2):
        pre = f"model.layers.{l}."
        for got, key in ((base.q[l], "self_attn.q_proj"), (base.k[l], "self_attn.k_proj"),
                         (base.v[l], "self_attn.v_proj"), (base.o[l], "self_attn.o_proj"),
                         (base.gate[l], "mlp.gate_proj"), (base.up[l], "mlp.up_proj"),
                         (base.down[l], "mlp.down_proj"), (base.in_norm[l], "input_layernorm"),
                         (base.post_norm[l], "post_attention_layernorm")):
            assert got.dtype == BF and torch.equal(got, sd[pre + key + ".weight"]), (l, key)
    assert torch.equal(base.embed, sd["model.embed_tokens.weight"])
    assert torch.equal(base.final_norm, sd["model.norm.weight"])
    assert torch.equal(base.lm_head, sd["lm_head.weight"] if not tie else sd["model.embed_tokens.weight"])


def test_config_of_either_transformers_generation():
    v4 = {"hidden_size": 64, "intermediate_size": 96, "num_hidden_layers": 2, "num_attention_heads": 2,
          "num_key_value_heads": 1, "vocab_size": 128, "rope_theta": 500000.0,
          "rope_scaling": {"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                           "original_max_position_embeddings": 8192, "rope_type": "llama3"}}
    v5 = {k: v for k, v in v4.items() if k not in ("rope_theta", "rope_scaling")}
    v5["rope_parameters"] = dict(v4["rope_scaling"], rope_theta=500000.0)
    a, b = ck.config_from_hf(v4), ck.config_from_hf(v5)
    assert a == b and a.rope_theta == 500000.0 and a.rope_scaling == v4["rope_scaling"]
    plain = dict(v5, rope_parameters={"rope_type": "default", "rope_theta": 10000.0})
    assert ck.config_from_hf(plain).rope_scaling == {}


def test_config_defaults_follow_the_reference():
    cfg = ck.config_from_hf({"hidden_size": 4096, "intermediate_size": 14336, "num_hidden_layers": 32,
                             "num_attention_heads": 32, "vocab_size": 128256}, rank=32)
    assert cfg.hkv == 32 and cfg.head_dim == 128 and cfg.eps == 1e-6 and cfg.rank == 32
    assert cfg.rope_scaling == {} and cfg.rope_theta == 10000.0


def test_refuses_broken_checkpoints(scratch):
    model, d = _tiny(False, scratch, "broken", "10GB")
    cfg = json.loads((d / "config.json").read_text())
    cfg["intermediate_size"] = 128
    (d / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(ValueError, match="shape"):
        ck.load_base(str(d), "cpu")
    (d / "model.safetensors").rename(d / "pytorch_model.bin")
    with pytest.raises(ValueError, match="pickled"):
        ck.load_base(str(d), "cpu")
    (d / "pytorch_model.bin").unlink()
    with pytest.raises(FileNotFoundError):
        ck.load_base(str(d), "cpu")
