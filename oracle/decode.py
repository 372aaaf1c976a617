"""CPU restatement of one decode token for N slots (test infrastructure).

Follows the worker's per-token loop (src/worker/worker_sync.py:1274-1425)
with the aggregator's rounds (src/cpp_extensions/ext_aggregator.cpp:470-875)
for every slot, using the arithmetic of oracle.reference_math. State (KV
caches, positions) is mutated in place like the reference's PagedKVCache.
"""
from __future__ import annotations

import math

import torch

from . import reference_math as ref


def decode_step(cfg, base, adapters, k_cache, v_cache, block_tables, seqlens, tokens):
    """One step for every slot: tokens[i] is one token id, or a list of ids
    (several new rows, e.g. a prefill chunk, at positions seqlens[i] ..
    seqlens[i] + len - 1; the rows of a slot attend causally to each other).

    base: object with CPU bf16 lists q,k,v,o,gate,up,down,in_norm,post_norm and
    tensors final_norm, embed, lm_head (HF [out, in] layout).
    adapters[i][layer][name] = (lora_A [r, in], lora_B [out, r]) or None; each
    adapter's scaling is cfg.alpha / its own rank (load_lora_fast,
    model_builder.py:147-149), so adapters of different ranks can share a step.
    k_cache/v_cache[layer]: [pages, page, hkv, D] (shared page pool).
    Returns (next_tokens [N] int64, final normed hidden [N, H], logits [N, vocab],
    last-layer hidden before the final norm [N, H]), all from each slot's
    last row.
    """
    n = len(tokens)
    D = cfg.head_dim

    def scaling(ad):
        return cfg.alpha / int(ad["q"][0].shape[0])

    scale = 1.0 / math.sqrt(D)
    ids = [torch.tensor(list(t) if isinstance(t, (list, tuple)) else [t]) for t in tokens]
    h = ref.embed_round(ids, base.embed)  # list of [1, H]
    qkv_dims = [cfg.hq * D, cfg.hkv * D, cfg.hkv * D]
    for l in range(cfg.layers):
        residual = h
        x = [ref.rms_norm(hi, base.in_norm[l], cfg.eps) for hi in h]
        qkv_base = ref.slot_round(x, ref.fuse_qkv(base.q[l], base.k[l], base.v[l]))
        attn_out = []
        for i in range(n):
            parts = list(torch.split(qkv_base[i], qkv_dims, -1))
            ad = adapters[i][l] if adapters[i] is not None else None
            if ad is not None:
                fA, fB = ref.pack_fused_lora([ad[p][0] for p in ("q", "k", "v")],
                                             [ad[p][1] for p in ("q", "k", "v")], scaling(ad), qkv_dims)
                parts = [ref.add_bf16(p, d) for p, d in
                         zip(parts, ref.fused_lora_delta(x[i], fA, fB, qkv_dims))]
            T = x[i].shape[0]
            pos = torch.arange(seqlens[i], seqlens[i] + T)
            cs = ref.cos_sin_cache(ref.llama3_inv_freq(D), seqlens[i] + T)
            q = ref.rope_neox(parts[0], pos, cs, D)
            k = ref.rope_neox(parts[1], pos, cs, D)
            o = ref.attention_with_kvcache(q.reshape(T, cfg.hq, D), k.reshape(T, cfg.hkv, D),
                                           parts[2].reshape(T, cfg.hkv, D), k_cache[l], v_cache[l],
                                           block_tables[i], seqlens[i], scale)
            attn_out.append(o.reshape(T, cfg.hq * D))
        o_base = ref.slot_round(attn_out, base.o[l])
        h = []
        for i in range(n):
            o = o_base[i]
            ad = adapters[i][l] if adapters[i] is not None else None
            if ad is not None:
                o = ref.add_bf16(o, ref.lora_delta_scale_after(attn_out[i], ad["o"][0], ad["o"][1], scaling(ad)))
            h.append(ref.add_bf16(residual[i], o))
        mlp_res = h
        x = [ref.rms_norm(hi, base.post_norm[l], cfg.eps) for hi in h]
        gu_base = ref.slot_round(x, ref.fuse_gate_up(base.gate[l], base.up[l]))
        act = []
        for i in range(n):
            gate, up = torch.split(gu_base[i], [cfg.inter, cfg.inter], -1)
            ad = adapters[i][l] if adapters[i] is not None else None
            if ad is not None:
                fA, fB = ref.pack_fused_lora([ad["gate"][0], ad["up"][0]], [ad["gate"][1], ad["up"][1]],
                                             scaling(ad), [cfg.inter, cfg.inter])
                dg, du = ref.fused_lora_delta(x[i], fA, fB, [cfg.inter, cfg.inter])
                gate, up = ref.add_bf16(gate, dg), ref.add_bf16(up, du)
            act.append(ref.silu_mul(gate, up))
        d_base = ref.slot_round(act, base.down[l])
        h = []
        for i in range(n):
            d = d_base[i]
            ad = adapters[i][l] if adapters[i] is not None else None
            if ad is not None:
                d = ref.add_bf16(d, ref.lora_delta_scale_after(act[i], ad["down"][0], ad["down"][1], scaling(ad)))
            h.append(ref.add_bf16(mlp_res[i], d))
    final = torch.cat([ref.rms_norm(hi[-1:], base.final_norm, cfg.eps) for hi in h], 0)
    logits = ref.lm_head_logits(final, base.lm_head)
    return ref.greedy(logits), final, logits, torch.cat([hi[-1:] for hi in h], 0)
