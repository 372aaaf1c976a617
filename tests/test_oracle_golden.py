"""The CPU oracle against the golden fixtures made by running the reference's
own Python code (tests/golden/make_golden.py), and against HF transformers'
Llama decoder as an independent check of the layer glue. CPU only.

Bit-exact where the oracle restates the same bf16 operations; the HF check
uses the tolerances of tests/tolerances.py (HF rounds attention internals at
other points than flash-attention does).
"""
import math
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

from oracle import reference_math as ref
from oracle.decode import decode_step

GOLDEN = Path(__file__).resolve().parent / "golden"
BF = torch.bfloat16


def _load(name):
    return torch.load(GOLDEN / name, weights_only=False)


@pytest.mark.parametrize("case", ["qkv", "qkv_missing_k", "gate_up"])
def test_fused_lora_matches_reference(case):
    """FusedLoRA packing and forward (model_builder.py:217-262)."""
    c = _load("fused_lora.pt")[case]
    As, Bs = c["As"], c["Bs"]
    if c["missing"]:
        # a projection without adapter contributes zero A columns / B rows
        As = [torch.zeros_like(a) if i in c["missing"] else a for i, a in enumerate(As)]
        Bs = [torch.zeros_like(b) if i in c["missing"] else b for i, b in enumerate(Bs)]
    fA, fB = ref.pack_fused_lora(As, Bs, c["scaling"], c["out_dims"])
    assert torch.equal(fA, c["fused_A"])
    assert torch.equal(fB, c["fused_B"])
    for got, want in zip(ref.fused_lora_delta(c["x"], fA, fB, c["out_dims"]), c["deltas"]):
        assert torch.equal(got, want)


@pytest.mark.parametrize("case", ["o", "down"])
def test_scale_after_lora_and_residual_match_reference(case):
    """O / Down LoRA (worker_sync.py:305, :375) and the residual adds."""
    c = _load("lora_scale_after.pt")[case]
    d = ref.lora_delta_scale_after(c["x"], c["A"], c["B"], c["scaling"])
    assert torch.equal(d, c["delta"])
    assert torch.equal(ref.add_bf16(c["residual"], ref.add_bf16(c["raw"], d)), c["hidden"])


def test_cos_sin_cache_matches_reference():
    """build_vllm_cos_sin_cache over the Llama-3.1 rotary module."""
    c = _load("cos_sin_cache.pt")
    inv = ref.llama3_inv_freq()
    assert torch.allclose(inv, c["inv_freq"], rtol=1e-6, atol=0)
    assert torch.equal(ref.cos_sin_cache(c["inv_freq"], c["max_seq_len"]), c["cache"])


def test_paged_kv_bookkeeping_matches_reference():
    """PagedKVCache allocation, advance, zero-on-free (paged_attention.py:7-128)."""
    c = _load("paged_kv_cache.pt")
    kv = ref.PagedKV(num_layers=2, num_blocks=c["num_blocks"], block_size=c["block_size"], kv_heads=2,
                     head_dim=8)
    for (op, slot, arg), snap in zip(c["script"], c["snaps"]):
        if op == "ensure":
            kv.ensure(slot, arg)
        elif op == "advance":
            kv.seq_lens[slot] += arg
        elif op == "free":
            kv.free_slot(slot)
        elif op == "fill":
            b = kv.tables[slot][0]
            for layer in range(2):
                kv.k[layer][b].fill_(arg)
                kv.v[layer][b].fill_(arg)
        live = sorted(kv.tables)
        assert live == snap["slots"]
        assert kv.free == snap["free"]
        assert [float(k.float().sum()) for k in kv.k] == snap["k_sum"]
        if live:
            width = snap["tables"].shape[1]
            tables = torch.zeros(len(live), width, dtype=torch.int32)
            for i, s in enumerate(live):
                tables[i, :len(kv.tables[s])] = torch.tensor(kv.tables[s], dtype=torch.int32)
            assert torch.equal(tables, snap["tables"])
            assert [kv.seq_lens[s] for s in live] == snap["seq_lens"].tolist()


def test_decode_step_matches_hf_llama():
    """One-layer model: the oracle's incremental decode (paged KV, NeoX RoPE,
    GQA attention, RMSNorm, SiLU MLP, greedy LM head) against HF
    LlamaForCausalLM run over the whole sequence on CPU."""
    from transformers import LlamaConfig, LlamaForCausalLM
    H, I, D, hq, hkv, V, P = 256, 512, 128, 2, 1, 64, 24
    hf_cfg = LlamaConfig(hidden_size=H, intermediate_size=I, num_attention_heads=hq, num_key_value_heads=hkv,
                         head_dim=D, num_hidden_layers=1, vocab_size=V, rms_norm_eps=1e-5,
                         rope_theta=500000.0, max_position_embeddings=131072, tie_word_embeddings=False,
                         rope_scaling={"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                       "original_max_position_embeddings": 8192, "rope_type": "llama3"},
                         attn_implementation="eager")
    torch.manual_seed(7)
    model = LlamaForCausalLM(hf_cfg).to(BF).eval()
    g = torch.Generator().manual_seed(8)
    with torch.no_grad():
        for p in model.parameters():
            p.copy_((torch.randn(p.shape, generator=g) * 0.05).to(BF))
        for norm in (model.model.layers[0].input_layernorm, model.model.layers[0].post_attention_layernorm,
                     model.model.norm):
            norm.weight.copy_((1 + 0.1 * torch.randn(H, generator=g)).to(BF))
    lay = model.model.layers[0]
    base = SimpleNamespace(q=[lay.self_attn.q_proj.weight], k=[lay.self_attn.k_proj.weight],
                           v=[lay.self_attn.v_proj.weight], o=[lay.self_attn.o_proj.weight],
                           gate=[lay.mlp.gate_proj.weight], up=[lay.mlp.up_proj.weight],
                           down=[lay.mlp.down_proj.weight], in_norm=[lay.input_layernorm.weight],
                           post_norm=[lay.post_attention_layernorm.weight], final_norm=model.model.norm.weight,
                           embed=model.model.embed_tokens.weight, lm_head=model.lm_head.weight)
    base = SimpleNamespace(**{k: ([t.detach() for t in v] if isinstance(v, list) else v.detach())
                              for k, v in vars(base).items()})
    cfg = SimpleNamespace(alpha=32, rank=16, head_dim=D, hq=hq, hkv=hkv, layers=1, inter=I, eps=1e-5)
    tokens = torch.randint(0, V, (P,), generator=g).tolist()
    kv = ref.PagedKV(num_layers=1, num_blocks=4, kv_heads=hkv, head_dim=D)
    kv.ensure(0, P)
    for pos in range(P):
        nxt, final, logits, _ = decode_step(cfg, base, [None], kv.k, kv.v, [kv.tables[0]], [pos], [tokens[pos]])
    with torch.no_grad():
        out = model(torch.tensor([tokens]), output_hidden_states=True)
    hf_final = out.hidden_states[-1][0, -1:]
    hf_logits = out.logits[0, -1:]
    err = (final.float() - hf_final.float()).norm() / hf_final.float().norm()
    assert err < 2e-2, f"final hidden relative error {err:.3e}"
    lerr = (logits.float() - hf_logits.float()).norm() / hf_logits.float().norm()
    assert lerr < 2e-2, f"logits relative error {lerr:.3e}"
    top = hf_logits.float().max()
    assert hf_logits[0, int(nxt[0])].float() >= top - 2.0 ** -7 * top.abs() - 1e-3


@pytest.mark.parametrize("r", [4, 8, 16, 32])  # 4: the reference's adapter generator mixes rank-4 adapters in
def test_rank_padding_and_scale_folding_are_exact(r):
    """A group runs every adapter at its largest rank R: lora_A / lora_B get
    zero rows / columns, and an O/Down adapter's own scale alpha/r is folded
    into its lora_B as (alpha/r) / (alpha/R) so the kernels apply one scale
    per launch. Through the oracle's scale-after LoRA (worker_sync.py:305,
    :375) both are bit-identical to the adapter at its own rank."""
    alpha, R, K, N = 32, 32, 512, 256
    g = torch.Generator().manual_seed(r)
    x = torch.randn(3, K, generator=g).to(BF)
    A = (torch.randn(r, K, generator=g) * 0.02).to(BF)
    B = (torch.randn(N, r, generator=g) * 0.02).to(BF)
    want = ref.lora_delta_scale_after(x, A, B, alpha / r)
    A_pad = torch.nn.functional.pad(A, (0, 0, 0, R - r))
    B_pad = torch.nn.functional.pad((B.float() * ((alpha / r) / (alpha / R))).to(BF), (0, R - r))
    got = ref.lora_delta_scale_after(x, A_pad, B_pad, alpha / R)
    assert torch.equal(got, want)
