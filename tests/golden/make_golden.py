"""Generates the golden fixtures in this directory by running the reference's
own Python code for the hot path's worker-side arithmetic (on CPU):

  * FusedLoRA (src/worker/model_builder.py:217-262) for the QKV and Gate+Up
    LoRA groups, including a group with one projection without adapter;
  * the O / Down LoRA path: SyncRemoteLoRALinear over FastLoRAModule
    (model_builder.py:31-46, :193-201) called as in
    src/worker/worker_sync.py:305 and :375, then the residual adds of
    worker_sync.py:311-319 / :381-389;
  * build_vllm_cos_sin_cache (src/worker/paged_attention.py:131-142) over the
    Llama-3.1 LlamaRotaryEmbedding (the worker's rotary module,
    model_builder.py:293-303);
  * PagedKVCache block bookkeeping (paged_attention.py:7-128) on a scripted
    sequence of allocations, frees and advances;
  * two tiny adapter directories written by the reference's adapter
    generator (generate_adapters.py:65-129: fp32 safetensors in the PEFT
    layout), one with every projection at alpha = r, one at rank 8 with
    lora_alpha 16 and without v_proj / down_proj, and what the reference's
    loader (model_builder.py:137-183, load_lora_fast) reads from them.

Run from the repository root where the reference checkout is available:
    python tests/golden/make_golden.py /path/to/reference
It needs the reference sources only at generation time; the fixtures it
writes (*.pt, a few hundred KB in total) are what the tests read. The native
module ext_unified_barrier is replaced by a stub holding its op constants
(the reference imports it at module load for those constants only).
"""
from __future__ import annotations

import sys

sys.dont_write_bytecode = True  # never write into the reference checkout
import types
from pathlib import Path

import torch

OUT = Path(__file__).resolve().parent
BF = torch.bfloat16


def _import_reference(ref_root: Path):
    stub = types.ModuleType("ext_unified_barrier")
    for name, val in (("OP_O_PROJ", 3), ("OP_DOWN_PROJ", 6), ("OP_QKV_FUSED", 9),
                      ("OP_GATE_UP_FUSED", 10), ("OP_EMBED", 11), ("OP_LM_HEAD", 12)):
        setattr(stub, name, val)
    sys.modules["ext_unified_barrier"] = stub
    sys.path.insert(0, str(ref_root / "src"))
    from worker import model_builder, paged_attention  # noqa: E402
    return model_builder, paged_attention


def _rnd(g, *shape, std=0.02):
    return (torch.randn(*shape, generator=g) * std).to(BF)


def fused_lora_case(mb, g, in_dim, out_dims, r, scaling, T, missing=()):
    As = [_rnd(g, r, in_dim) for _ in out_dims]
    Bs = [_rnd(g, d, r) for d in out_dims]
    mods = [None if i in missing else mb.FastLoRAModule(A, B, scaling) for i, (A, B) in enumerate(zip(As, Bs))]
    fl = mb.FusedLoRA(mods, list(out_dims), "cpu", BF)
    x = _rnd(g, T, in_dim, std=1.0)
    with torch.no_grad():
        deltas = fl(x)
    return {"As": As, "Bs": Bs, "missing": list(missing), "scaling": scaling, "out_dims": list(out_dims),
            "x": x, "fused_A": fl.fused_A.detach().clone(), "fused_B": fl.fused_B.detach().clone(),
            "deltas": [d.clone() for d in deltas]}


def scale_after_case(mb, g, in_dim, out_dim, r, scaling, T):
    A, B = _rnd(g, r, in_dim), _rnd(g, out_dim, r)
    m = mb.SyncRemoteLoRALinear(3, 0, out_dim, mb.FastLoRAModule(A, B, scaling))
    x = _rnd(g, T, in_dim, std=1.0)
    raw = _rnd(g, T, out_dim, std=1.0)
    residual = _rnd(g, T, out_dim, std=1.0)
    with torch.no_grad():
        delta = m.lora_B(m.lora_A(m.dropout(x))) * m.scaling  # worker_sync.py:305
        result = raw + delta                                   # worker_sync.py:316
        hidden = residual + result                             # worker_sync.py:319
    return {"A": A, "B": B, "scaling": scaling, "x": x, "raw": raw, "residual": residual,
            "delta": delta.clone(), "hidden": hidden.clone()}


def cos_sin_case(pa, max_seq_len):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    cfg = LlamaConfig(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8, rope_theta=500000.0,
                      max_position_embeddings=131072,
                      rope_scaling={"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                    "original_max_position_embeddings": 8192, "rope_type": "llama3"})
    rot = LlamaRotaryEmbedding(config=cfg)
    cache = pa.build_vllm_cos_sin_cache(rot, max_seq_len, "cpu", BF)
    return {"inv_freq": rot.inv_freq.float().clone(), "cache": cache.clone(), "max_seq_len": max_seq_len}


# (op, slot, arg): "ensure" -> ensure_blocks_for_length(slot, arg);
# "advance" -> advance_seq_lens([slot], arg); "free" -> free_slot(slot);
# "fill" -> fill the slot's first block with arg (to see the zeroing on free)
PAGED_SCRIPT = [("ensure", 0, 37), ("ensure", 1, 16), ("ensure", 2, 1), ("advance", 0, 37),
                ("advance", 1, 16), ("fill", 1, 3.0), ("ensure", 1, 17), ("free", 0, 0),
                ("ensure", 3, 40), ("ensure", 2, 33), ("advance", 2, 5), ("free", 1, 0), ("ensure", 0, 64)]


def paged_case(pa):
    c = pa.PagedKVCache(num_layers=2, num_kv_heads=2, head_dim=8, block_size=16, max_slots=4,
                        max_seq_len=64, device="cpu", dtype=BF)
    snaps = []
    for op, slot, arg in PAGED_SCRIPT:
        if op == "ensure":
            c.ensure_blocks_for_length(slot, arg)
        elif op == "advance":
            c.advance_seq_lens([slot], arg)
        elif op == "free":
            c.free_slot(slot)
        elif op == "fill":
            b = c.slot_block_tables[slot][0]
            for layer in range(c.num_layers):
                c.key_caches[layer][b].fill_(arg)
                c.value_caches[layer][b].fill_(arg)
        live = sorted(c.slot_block_tables)
        snaps.append({"slots": live,
                      "tables": c.get_block_table_tensor(live).clone() if live else torch.zeros(0),
                      "seq_lens": c.get_seq_lens_tensor(live).clone() if live else torch.zeros(0),
                      "free": list(c.free_blocks),
                      "k_sum": [float(k.float().sum()) for k in c.key_caches]})
    return {"num_blocks": c.num_blocks, "block_size": 16, "script": PAGED_SCRIPT, "snaps": snaps}


# (in_features, out_features) of a 2-layer model with hidden 64, 2 / 1
# heads of 32, intermediate 96 (engine.ModelConfig(hidden=64, inter=96,
# layers=2, hq=2, hkv=1, head_dim=32))
TINY_MODULES = {"self_attn.q_proj": (64, 64), "self_attn.k_proj": (64, 32), "self_attn.v_proj": (64, 32),
                "self_attn.o_proj": (64, 64), "mlp.gate_proj": (64, 96), "mlp.up_proj": (64, 96),
                "mlp.down_proj": (96, 64)}


def adapter_cases(mb, ref_root: Path):
    import importlib.util
    import json
    from safetensors.torch import save_file
    spec = importlib.util.spec_from_file_location("ref_generate_adapters", ref_root / "generate_adapters.py")
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    partial = {k: v for k, v in TINY_MODULES.items() if k not in ("self_attn.v_proj", "mlp.down_proj")}
    out = {}
    for name, rank, alpha, mods, seed in (("adapter_r4", 4, None, TINY_MODULES, 11),
                                          ("adapter_r8_partial", 8, 16, partial, 12)):
        d = OUT / name
        d.mkdir(exist_ok=True)
        save_file(gen.generate_adapter(rank, seed=seed, num_layers=2, modules=mods),
                  str(d / "adapter_model.safetensors"))
        cfg = gen.make_config(rank)
        if alpha is not None:
            cfg["lora_alpha"] = alpha
        cfg["target_modules"] = sorted({k.split(".")[1] for k in mods})
        (d / "adapter_config.json").write_text(json.dumps(cfg, indent=2))
        loaded, config = mb.load_lora_fast(str(d), "cpu", BF)
        out[name] = {"r": config["r"], "lora_alpha": config.get("lora_alpha", config["r"]),
                     "modules": {(layer, mod): (m.lora_A["default"].weight.detach().clone(),
                                                m.lora_B["default"].weight.detach().clone(),
                                                float(m.scaling["default"]))
                                 for layer, ms in loaded.items() for mod, m in ms.items()}}
    return out


def main(ref_root: str) -> None:
    mb, pa = _import_reference(Path(ref_root))
    torch.save(adapter_cases(mb, Path(ref_root)), OUT / "adapter_load.pt")
    g = torch.Generator().manual_seed(20261201)
    torch.save({"qkv": fused_lora_case(mb, g, 256, (256, 64, 64), 8, 2.0, 3),
                "qkv_missing_k": fused_lora_case(mb, g, 256, (256, 64, 64), 8, 2.0, 2, missing=(1,)),
                "gate_up": fused_lora_case(mb, g, 256, (512, 512), 8, 2.0, 2)}, OUT / "fused_lora.pt")
    torch.save({"o": scale_after_case(mb, g, 256, 256, 8, 2.0, 3),
                "down": scale_after_case(mb, g, 512, 256, 16, 2.0, 2)}, OUT / "lora_scale_after.pt")
    torch.save(cos_sin_case(pa, 320), OUT / "cos_sin_cache.pt")
    torch.save(paged_case(pa), OUT / "paged_kv_cache.pt")
    for f in sorted(OUT.glob("*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")
