"""End to end against an independent implementation: a two-layer Llama at
the 8B layer shapes, written by transformers (save_pretrained, the format
the reference's aggregator loads), loaded with swarmlora_b200.checkpoint and
run through the engine (aggregator rounds + worker kernels, no adapter):
the prompt is prefilled in 16-row chunks, then tokens are decoded one step
at a time. At every decode step the last row's hidden state before the final
norm matches the reference's arithmetic (the CPU oracle) at the multi-layer
tolerance and HF LlamaForCausalLM's fp32 forward within the 2e-2 relative
bar; the picked token is the oracle's and within rounding of HF's maximum.
The engine's own tokens are fed to all three, so the sequences never
diverge."""
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


def _rel_fro(got: torch.Tensor, ref: torch.Tensor) -> float:
    g, r = got.detach().float().cpu().flatten(), ref.detach().float().cpu().flatten()
    return float((g - r).norm() / r.norm())


def test_engine_matches_hf_llama_from_a_checkpoint(native, cuda, scratch):
    """Two checks per step, on the last row's hidden state before the final
    norm and on the picked token:

    * parity: the engine against the reference's own arithmetic (the CPU
      oracle) on the same checkpoint, chunks and tokens, at the multi-layer
      tolerance;
    * independence: the engine against HF LlamaForCausalLM run in fp32 on the
      same bf16 weights (the exact model), within the 2e-2 relative Frobenius
      bar, and no further from it than the reference's arithmetic is (1.25x
      the oracle's own distance, plus 2e-3 for summation order).

    HF's bf16 eager forward is not the yardstick: it rounds attention scores
    and probabilities to bf16, and on this model it is 1.7e-2 to 2.1e-2 away
    from its own fp32 forward, with single elements up to 9% of the row rms;
    the reference's arithmetic itself misses an elementwise bound against it
    at most steps. Against fp32 HF the reference's arithmetic is 1.4e-2 to
    1.7e-2 away (bf16 activations through two 8B-shaped layers), so an
    elementwise bound against fp32 HF is not applied either."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from oracle.decode import decode_step
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
    base_c, _ = load_base(str(scratch / "llama2l"), "cpu")
    exact = LlamaForCausalLM(hf_cfg).eval()  # fp32 arithmetic on the same bf16 weights
    exact.load_state_dict({k: v.float() for k, v in model.state_dict().items()})
    del model
    pre_norm = {}
    exact.model.norm.register_forward_hook(lambda mod, inp, out: pre_norm.__setitem__("h", inp[0].detach()))

    g = torch.Generator().manual_seed(12)
    prompt = torch.randint(0, cfg.vocab, (20,), generator=g).tolist()
    grp = SlotGroup(cfg, base, [None], [0], max_new=48, seed=0)
    try:
        kc = [k.cpu() for k in grp.k_cache]
        vc = [v.cpu() for v in grp.v_cache]
        bts = [t.tolist() for t in grp.block_tables]
        stream = torch.cuda.current_stream()
        seq = list(prompt)
        done = 0
        seqlen = 0
        checked = 0
        for step in range(8):
            if done < len(prompt):  # prefill chunks of up to 16 rows
                rows = min(16, len(prompt) - done)
                toks = prompt[done:done + rows]
                grp.enqueue_step(stream, rows=[rows], tokens=[toks])
                done += rows
            else:
                rows = 1
                toks = [seq[-1]]
                grp.tokens.copy_(torch.tensor(toks))
                grp.enqueue_step(stream)
            torch.cuda.synchronize()
            want, _, o_logits, o_h = decode_step(cfg, base_c, [None], kc, vc, bts, [seqlen], [toks])
            seqlen += rows
            if done < len(prompt):
                continue
            got_h = grp.h_rows[0, rows - 1].reshape(1, -1)
            assert_close(got_h, o_h, f"step {step}: last hidden before the final norm vs the oracle",
                         atol_rms=ATOL_RMS_MULTILAYER)
            tok = int(grp.tokens[0])
            lo = o_logits[0].float()
            assert tok == int(want[0]) or lo[tok] >= lo.max() - 2.0 ** -8 * lo.max().abs(), \
                f"step {step}: token {tok} != oracle {int(want[0])}"
            with torch.no_grad():
                out = exact(torch.tensor([seq]))
            h_exact = pre_norm["h"][0, -1:]
            e_engine, e_oracle = _rel_fro(got_h, h_exact), _rel_fro(o_h, h_exact)
            assert e_engine <= 2e-2, f"step {step}: {e_engine:.3e} from fp32 HF (bar 2e-2)"
            assert e_engine <= 1.25 * e_oracle + 2e-3, \
                f"step {step}: {e_engine:.3e} from fp32 HF, the reference's arithmetic {e_oracle:.3e}"
            logits = out.logits[0, -1].float()
            top = logits.max()
            # the engine's hidden differs from the exact one by bf16 rounding
            # (about 1.5% of its norm), so accept a token within 5% of the
            # logits' spread of HF's maximum
            tol = 2.0 ** -7 * top.abs() + 0.05 * logits.std()
            assert logits[tok] >= top - tol, f"step {step}: token {tok} is {float(top - logits[tok]):.4f} below HF's max"
            seq.append(tok)
            checked += 1
        assert checked == 7
    finally:
        grp.close()
