"""End to end against an independent implementation: a two-layer Llama at
the 8B layer shapes, written by transformers (save_pretrained, the format
the reference's aggregator loads), loaded with swarmlora_b200.checkpoint and
run through the engine (aggregator rounds + worker kernels, no adapter):
the prompt is prefilled in 16-row chunks, then tokens are decoded one step
at a time. At every step the last row's hidden state before the final norm
matches HF LlamaForCausalLM's (run over the whole sequence on the CPU)
within the multi-layer tolerance, and the picked token's HF logit is within
the two implementations' rounding difference of HF's maximum; HF's token is
fed to both so the sequences never diverge."""
import pytest
import torch

from tests.tolerances import ATOL_RMS_MULTILAYER, assert_close

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def test_loaders_on_the_device_equal_their_cpu_loads(native, cuda, scratch):
    """The adapter and checkpoint loaders through the pinned staging buffer
    and the asynchronous host-to-device copies (the staging buffer reused
    across tensors and across loads) give exactly what they give on the CPU."""
    from pathlib import Path
    from transformers import LlamaConfig, LlamaForCausalLM
    from swarmlora_b200 import adapters as ad
    from swarmlora_b200.checkpoint import load_base
    from swarmlora_b200.engine import ModelConfig
    golden = Path(__file__).resolve().parent / "golden"
    tiny = ModelConfig(hidden=64, inter=96, layers=2, hq=2, hkv=1, head_dim=32, vocab=128)
    loader = ad.AdapterLoader(tiny, cuda)
    for name in ("adapter_r4", "adapter_r8_partial", "adapter_r4"):
        on_dev, cfg_d = loader.load(str(golden / name))
        on_cpu, cfg_c = ad.load_adapter(str(golden / name), tiny, "cpu")
        assert cfg_d == cfg_c
        for l in range(tiny.layers):
            for p in ad.MODULES:
                for a, b in zip(on_dev[l][p], on_cpu[l][p]):
                    assert a.is_cuda and torch.equal(a.cpu(), b), (name, l, p)
    hf = LlamaConfig(hidden_size=64, intermediate_size=96, num_attention_heads=2, num_key_value_heads=1,
                     head_dim=32, num_hidden_layers=2, vocab_size=128, tie_word_embeddings=False)
    LlamaForCausalLM(hf).to(BF).save_pretrained(str(scratch / "tiny"), safe_serialization=True,
                                                max_shard_size="20KB")
    dev_base, _ = load_base(str(scratch / "tiny"), cuda)
    cpu_base, _ = load_base(str(scratch / "tiny"), "cpu")
    for field in ("q", "k", "v", "o", "gate", "up", "down", "in_norm", "post_norm"):
        for a, b in zip(getattr(dev_base, field), getattr(cpu_base, field)):
            assert a.is_cuda and torch.equal(a.cpu(), b), field
    for field in ("final_norm", "embed", "lm_head"):
        assert torch.equal(getattr(dev_base, field).cpu(), getattr(cpu_base, field)), field


def test_engine_matches_hf_llama_from_a_checkpoint(native, cuda, scratch):
    from transformers import LlamaConfig, LlamaForCausalLM
    from swarmlora_b200.checkpoint import load_base
    from swarmlora_b200.engine import SlotGroup
    hf_cfg = LlamaConfig(hidden_size=4096, intermediate_size=14336, num_attention_heads=32, num_key_value_heads=8,
                         head_dim=128, num_hidden_layers=2, vocab_size=4096, rms_norm_eps=1e-5,
                         rope_theta=500000.0, max_position_embeddings=131072, tie_word_embeddings=False,
                         rope_scaling={"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                       "original_max_position_embeddings": 8192, "rope_type": "llama3"},
                         attn_implementation="eager")
    torch.manual_seed(11)
    model = LlamaForCausalLM(hf_cfg).to(BF).eval()
    with torch.no_grad():
        for layer in model.model.layers:
            layer.input_layernorm.weight.copy_(1 + 0.1 * torch.randn(4096))
            layer.post_attention_layernorm.weight.copy_(1 + 0.1 * torch.randn(4096))
    model.save_pretrained(str(scratch / "llama2l"), safe_serialization=True)
    base, cfg = load_base(str(scratch / "llama2l"), cuda)
    pre_norm = {}
    model.model.norm.register_forward_hook(lambda mod, inp, out: pre_norm.__setitem__("h", inp[0].detach()))

    g = torch.Generator().manual_seed(12)
    prompt = torch.randint(0, cfg.vocab, (20,), generator=g).tolist()
    grp = SlotGroup(cfg, base, [None], [0], max_new=48, seed=0)
    try:
        stream = torch.cuda.current_stream()
        seq = list(prompt)
        done = 0
        for step in range(8):
            if done < len(prompt):  # prefill chunks of up to 16 rows
                rows = min(16, len(prompt) - done)
                grp.enqueue_step(stream, rows=[rows], tokens=[prompt[done:done + rows]])
                done += rows
            else:
                rows = 1
                grp.tokens.copy_(torch.tensor([seq[-1]]))
                grp.enqueue_step(stream)
            torch.cuda.synchronize()
            if done < len(prompt):
                continue
            with torch.no_grad():
                out = model(torch.tensor([seq]))
            logits = out.logits[0, -1].float()
            assert_close(grp.h_rows[0, rows - 1].reshape(1, -1), pre_norm["h"][0, -1:],
                         f"step {step}: last hidden before the final norm", atol_rms=ATOL_RMS_MULTILAYER)
            tok = int(grp.tokens[0])
            top = logits.max()
            # HF rounds its attention to bf16 where the engine keeps fp32, so
            # the two logit vectors differ by about 1% of their spread: accept
            # a token within that of HF's maximum
            tol = 2.0 ** -7 * top.abs() + 0.05 * logits.std()
            assert logits[tok] >= top - tol, f"step {step}: token {tok} is {float(top - logits[tok]):.4f} below HF's max"
            seq.append(int(logits.argmax()))
        assert len(seq) > len(prompt) + 3
    finally:
        grp.close()
