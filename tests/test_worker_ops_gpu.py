"""Worker-side kernels against the CPU oracle.

LoRA delta + round epilogue in its three modes (QKV add, O/Down residual,
Gate+Up SiLU-mul), slots without an adapter, NeoX RoPE + paged KV append +
causal GQA attention with ragged contexts, prefill chunks and page-boundary
positions, and RMSNorm. Seeded inputs; adapters A, B ~ N(0, 0.02), r = 16,
alpha = 32.
"""
import math

import pytest
import torch

from oracle import reference_math as ref
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
BF = torch.bfloat16
H, I, HQ, HKV, D = 4096, 14336, 32, 8, 128
QKV_DIMS = [4096, 1024, 1024]


def _g(seed):
    return torch.Generator().manual_seed(seed)


def _adapter(g, in_dim, out_dim, r=16):
    A = (torch.randn(r, in_dim, generator=g) * 0.02).to(BF)
    B = (torch.randn(out_dim, r, generator=g) * 0.02).to(BF)
    return A, B


def _run_expand_case(mode, rows, seed, with_missing=False):
    from swarmlora_b200 import worker_ops as wo
    g = _g(seed)
    r, s = 16, 2.0
    if mode == wo.EXPAND_ADD:
        K, dims = H, QKV_DIMS
    elif mode == wo.EXPAND_SILU_MUL:
        K, dims = H, [I, I]
    else:
        K, dims = (H, [H]) if seed % 2 == 0 else (I, [H])
    n_total = sum(dims)
    xs = [torch.randn(n, K, generator=g).to(BF) for n in rows]
    bases = [torch.randn(n, n_total, generator=g).to(BF) for n in rows]
    resids = [torch.randn(n, H, generator=g).to(BF) for n in rows]
    adapters = []
    for i in range(len(rows)):
        if with_missing and i == 1:
            adapters.append(None)
        else:
            adapters.append([_adapter(g, K, d, r) for d in dims])
    # --- oracle
    want = []
    for i, n in enumerate(rows):
        ad = adapters[i]
        if mode == wo.EXPAND_RESIDUAL:
            o = bases[i]
            if ad is not None:
                o = ref.add_bf16(o, ref.lora_delta_scale_after(xs[i], ad[0][0], ad[0][1], s))
            want.append(ref.add_bf16(resids[i], o))
            continue
        if ad is not None:
            fA, fB = ref.pack_fused_lora([a for a, _ in ad], [b for _, b in ad], s, dims)
            deltas = ref.fused_lora_delta(xs[i], fA, fB, dims)
        else:
            deltas = [None] * len(dims)
        parts = list(torch.split(bases[i], dims, -1))
        parts = [p if d is None else ref.add_bf16(p, d) for p, d in zip(parts, deltas)]
        if mode == wo.EXPAND_ADD:
            want.append(torch.cat(parts, -1))
        else:
            want.append(ref.silu_mul(parts[0], parts[1]))
    # --- device
    R = r * len(dims)
    As, Bs = [], []
    for ad in adapters:
        if ad is None:
            As.append(None)
            Bs.append(None)
            continue
        if mode == wo.EXPAND_RESIDUAL:
            As.append(ad[0][0].t().contiguous().to(DEV))
        else:
            As.append(torch.cat([(a.t() * s).to(BF) for a, _ in ad], 1).contiguous().to(DEV))
        Bs.append(torch.cat([b for _, b in ad], 0).contiguous().to(DEV))
    xd = [x.to(DEV) for x in xs]
    bd = [b.to(DEV) for b in bases]
    rd = [x.to(DEV) for x in resids]
    n_out = n_total // 2 if mode == wo.EXPAND_SILU_MUL else n_total
    if mode == wo.EXPAND_RESIDUAL:
        n_out = H
    outs = [torch.empty(n, n_out, dtype=BF, device=DEV) for n in rows]
    splits = 4
    ws = torch.empty(splits * sum(rows) * R, dtype=torch.float32, device=DEV)
    wo.lora_shrink(xd, As, K, R, splits, ws)
    ends = list(torch.tensor(dims).cumsum(0).tolist())
    wo.lora_expand(bd, Bs, outs, n_total, r, ends, mode, splits, ws,
                   resids=rd if mode == wo.EXPAND_RESIDUAL else None,
                   post_scale=s if mode == wo.EXPAND_RESIDUAL else 0.0,
                   resid_stride=H)
    torch.cuda.synchronize()
    for i, (o, w) in enumerate(zip(outs, want)):
        assert_close(o, w, f"mode {mode} slot {i}")


@pytest.mark.parametrize("rows", [[1] * 6, [1, 16, 3, 1]])
def test_lora_qkv_add(native, cuda, rows):
    from swarmlora_b200 import worker_ops as wo
    _run_expand_case(wo.EXPAND_ADD, rows, seed=1)


@pytest.mark.parametrize("seed", [2, 3])  # even: O (K=4096), odd: Down (K=14336)
def test_lora_residual(native, cuda, seed):
    from swarmlora_b200 import worker_ops as wo
    _run_expand_case(wo.EXPAND_RESIDUAL, [1, 1, 5, 1], seed=seed)


def test_lora_gate_up_silu(native, cuda):
    from swarmlora_b200 import worker_ops as wo
    _run_expand_case(wo.EXPAND_SILU_MUL, [1, 2, 1], seed=4)


def test_lora_missing_adapter(native, cuda):
    from swarmlora_b200 import worker_ops as wo
    _run_expand_case(wo.EXPAND_ADD, [1, 1, 1], seed=5, with_missing=True)
    _run_expand_case(wo.EXPAND_RESIDUAL, [1, 1, 1], seed=6, with_missing=True)


def _attn_case(ctx, rows, seed, page=16):
    """ctx[i]: cached tokens of slot i before the step; rows[i]: new tokens."""
    from swarmlora_b200 import worker_ops as wo
    g = _g(seed)
    n = len(ctx)
    max_len = max(c + r for c, r in zip(ctx, rows))
    pages_per = (max_len + page - 1) // page + 1
    num_pages = n * pages_per
    perm = torch.randperm(num_pages, generator=g).tolist()
    tables = [perm[i * pages_per:(i + 1) * pages_per] for i in range(n)]
    kc = (torch.randn(num_pages, page, HKV, D, generator=g)).to(BF)
    vc = (torch.randn(num_pages, page, HKV, D, generator=g)).to(BF)
    qkv = [torch.randn(r, (HQ + 2 * HKV) * D, generator=g).to(BF) for r in rows]
    inv = ref.llama3_inv_freq()
    cs = ref.cos_sin_cache(inv, 4096)
    scale = 1.0 / math.sqrt(D)
    # --- oracle
    kc_ref, vc_ref = kc.clone(), vc.clone()
    want = []
    for i in range(n):
        pos = torch.arange(ctx[i], ctx[i] + rows[i])
        q = ref.rope_neox(qkv[i][:, :HQ * D], pos, cs, D)
        k = ref.rope_neox(qkv[i][:, HQ * D:(HQ + HKV) * D], pos, cs, D)
        v = qkv[i][:, (HQ + HKV) * D:]
        o = ref.attention_with_kvcache(q.reshape(-1, HQ, D), k.reshape(-1, HKV, D),
                                       v.reshape(-1, HKV, D), kc_ref, vc_ref, tables[i], ctx[i], scale)
        want.append(o.reshape(rows[i], HQ * D))
    # --- device
    kd, vd = kc.to(DEV), vc.to(DEV)
    bts = [torch.tensor(t, dtype=torch.int32, device=DEV) for t in tables]
    sls = [torch.tensor([c], dtype=torch.int32, device=DEV) for c in ctx]
    qkvd = [q.to(DEV) for q in qkv]
    total = sum(rows)
    q_rot = torch.empty(total, HQ * D, dtype=BF, device=DEV)
    nparts = wo.attention_part_floats(total, HQ, HKV, max_len)
    part = torch.empty(max(1, nparts), dtype=torch.float32, device=DEV)
    outs = [torch.empty(r, HQ * D, dtype=BF, device=DEV) for r in rows]
    csd = cs.to(DEV)
    wo.rope_append(qkvd, bts, [kd] * n, [vd] * n, sls, q_rot, csd, HQ, HKV)
    wo.paged_attention(rows, bts, [kd] * n, [vd] * n, sls, outs, q_rot, part, HQ, HKV, max_len, scale)
    torch.cuda.synchronize()
    assert torch.equal(kd.cpu(), kc_ref), "K cache append differs"
    assert torch.equal(vd.cpu(), vc_ref), "V cache append differs"
    for i in range(n):
        assert_close(outs[i], want[i], f"attention slot {i} ctx {ctx[i]} rows {rows[i]}")
    return [o.cpu() for o in outs]


@pytest.mark.parametrize("ctx,rows", [
    ([127, 0, 15, 16, 300], [1, 1, 1, 1, 1]),
    ([256, 1000, 513, 640], [1, 1, 1, 1]),
    ([0, 40, 7], [16, 16, 1]),
])
def test_rope_append_attention(native, cuda, ctx, rows):
    _attn_case(ctx, rows, seed=sum(ctx) + len(rows))


@pytest.mark.parametrize("ctx,rows,groups", [
    ([127, 0, 15, 16, 300, 1000], [1, 1, 1, 1, 1, 1], 0),  # decode rows, partial and empty last pages
    ([0, 40, 7, 300], [16, 15, 1, 2], 0),  # prefill chunks: rows paired on one page read
    ([1000, 3, 513, 77], [1, 4, 1, 16], 2),  # kv head groups split across CTAs
    ([4000, 33], [1, 3], 0),
])
def test_attention_tma_pages_match_lane_copies(native, cuda, ctx, rows, groups):
    """K/V pages loaded by TMA (one lane per warp, 128B-swizzled halves,
    the query rows by bulk copy, stale V rows past the causal end zeroed)
    and by per-lane cp.async copies give bit-identical outputs (the same
    values reach the same MMAs in the same order); against the oracle too."""
    from swarmlora_b200._native import check, lib
    try:
        check(lib().swl_attention_tune(0, 0, groups))
        check(lib().swl_attention_tma(1))
        tma = _attn_case(ctx, rows, seed=sum(ctx) + 11 * len(rows))
        check(lib().swl_attention_tma(0))
        copies = _attn_case(ctx, rows, seed=sum(ctx) + 11 * len(rows))
    finally:
        check(lib().swl_attention_tma(1))
        check(lib().swl_attention_tune(0, 0, 0))
    for i, (a, b) in enumerate(zip(tma, copies)):
        assert torch.equal(a, b), f"slot {i}: TMA pages differ from lane copies"


@pytest.mark.parametrize("ctx,rows", [
    ([4000, 1024, 2047, 3000, 1], [1, 1, 1, 1, 1]),  # the long-context configuration's range
    ([4000], [1]),  # one long row: 250 pages split over more pieces than the combine loads at once
    ([2000, 3040], [16, 16]),  # prefill chunks far into their prompts
])
def test_attention_long_contexts_and_many_pieces(native, cuda, ctx, rows):
    """Contexts up to 4000 tokens (the configurations with U[1024,4096] and
    U[256,2048] contexts), including a row whose pages are split over more
    pieces than the combine step reads in its first batch."""
    _attn_case(ctx, rows, seed=sum(ctx) + 7 * len(rows))


@pytest.mark.parametrize("ctx,rows", [([0, 40, 7, 300], [16, 15, 1, 2]), ([1000, 16, 0], [3, 16, 16])])
@pytest.mark.parametrize("pairing", [1, 0])
def test_attention_row_pairs_and_single_rows(native, cuda, ctx, rows, pairing):
    """Prefill chunks (several rows of one slot, even and odd counts) beside
    decode rows: with two rows of a slot sharing each page read and with
    every row reading alone, against the oracle."""
    from swarmlora_b200._native import check, lib
    try:
        check(lib().swl_attention_pairing(pairing))
        _attn_case(ctx, rows, seed=sum(ctx) + 3 * len(rows) + pairing)
    finally:
        check(lib().swl_attention_pairing(1))


@pytest.mark.parametrize("stages,groups", [(3, 2), (2, 2), (4, 4), (2, 8)])
def test_attention_head_groups_match_one_group(native, cuda, stages, groups):
    """CTAs that share a page's kv heads (each holding its group's slices,
    a smaller ring per CTA) give bit for bit the one-group result: every
    head still streams the same pages in the same order."""
    from swarmlora_b200 import worker_ops as wo
    g = _g(77)
    ctx, rows = [1000, 3, 513, 77, 0, 300], [1, 1, 1, 4, 16, 1]
    n, page = len(ctx), 16
    max_len = max(c + r for c, r in zip(ctx, rows))
    pages_per = (max_len + page - 1) // page + 1
    perm = torch.randperm(n * pages_per, generator=g).tolist()
    bts = [torch.tensor(perm[i * pages_per:(i + 1) * pages_per], dtype=torch.int32, device=DEV) for i in range(n)]
    kd = torch.randn(n * pages_per, page, HKV, D, generator=g).to(BF).to(DEV)
    vd = torch.randn(n * pages_per, page, HKV, D, generator=g).to(BF).to(DEV)
    sls = [torch.tensor([c], dtype=torch.int32, device=DEV) for c in ctx]
    total = sum(rows)
    q_rot = torch.randn(total, HQ * D, generator=g).to(BF).to(DEV)
    part = torch.empty(max(1, wo.attention_part_floats(total, HQ, HKV, max_len)), dtype=torch.float32, device=DEV)
    scale = 1.0 / math.sqrt(D)

    def run():
        outs = [torch.full((r, HQ * D), float("nan"), dtype=BF, device=DEV) for r in rows]
        wo.paged_attention(rows, bts, [kd] * n, [vd] * n, sls, outs, q_rot, part, HQ, HKV, max_len, scale)
        torch.cuda.synchronize()
        return [o.cpu() for o in outs]
    try:
        wo.attention_tune(0, 2, 1)
        want = run()
        wo.attention_tune(0, stages, groups)
        got = run()
    finally:
        wo.attention_tune(0, 0, 0)
    for i in range(n):
        assert torch.isfinite(want[i].float()).all()
        assert torch.equal(got[i], want[i]), f"slot {i}: {groups} head groups x {stages} stages differ"


def test_rope_matches_hf_rotary(native, cuda):
    """The oracle's llama3 inv_freq equals HF LlamaRotaryEmbedding's for Llama-3.1."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    cfg = LlamaConfig(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8,
                      rope_theta=500000.0,
                      rope_scaling={"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                    "original_max_position_embeddings": 8192, "rope_type": "llama3"})
    emb = LlamaRotaryEmbedding(config=cfg)
    assert torch.allclose(emb.inv_freq.float(), ref.llama3_inv_freq(), rtol=1e-6, atol=0)


@pytest.mark.parametrize("rows", [[1] * 7, [16, 1, 3]])
def test_rms_norm(native, cuda, rows):
    from swarmlora_b200 import worker_ops as wo
    g = _g(9)
    xs = [(torch.randn(r, H, generator=g) * 3).to(BF) for r in rows]
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(BF)
    outs = [torch.empty(r, H, dtype=BF, device=DEV) for r in rows]
    wo.rms_norm([x.to(DEV) for x in xs], outs, w.to(DEV), 1e-5)
    torch.cuda.synchronize()
    for x, o in zip(xs, outs):
        assert_close(o, ref.rms_norm(x, w, 1e-5), "rms_norm")
