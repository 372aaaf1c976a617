"""The fused round epilogues (worker_sync.py:1337-1409) called directly with
ragged token rows per slot (1, 16 and 3 rows: the packed prefill + decode
rows of the mixed configuration), against the oracle's arithmetic:

* swl_fused_resid_norm_shrink: O / Down LoRA expand scaled after, + residual,
  RMSNorm, and the next round's LoRA shrink partials;
* swl_fused_gu_silu_shrink: gate / up LoRA expand, SiLU * up, Down shrink
  partials;
* swl_fused_qkv_rope: q / k / v LoRA expand, NeoX RoPE at each row's
  position, rotated q and the new rows' K / V appended to the paged caches.

The LoRA intermediate t comes from seeded shrink partials (as the kernel
before each epilogue leaves them). Shapes are Llama-3.1-8B's, rank 16.
"""
import pytest
import torch

from oracle import reference_math as ref
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
H, I, D, HQ, HKV, R = 4096, 14336, 128, 32, 8, 16
ROWS = [1, 16, 3]
SPLITS_IN = 4


def _ptrs(native, ts):
    return native.ptr_array([t.data_ptr() if t is not None else None for t in ts])


def _t_from_partials(ws, n_cols):
    """bf16(sum over splits) per row, as the epilogues rebuild t."""
    return ref.bf(ws.view(-1, SPLITS_IN, n_cols).sum(1))


def _rand(g, *shape, std=1.0):
    return (torch.randn(*shape, generator=g) * std).to(BF)


def test_resid_norm_shrink_ragged_rows(native, cuda):
    lib = native.lib()
    g = torch.Generator().manual_seed(21)
    n, total = len(ROWS), sum(ROWS)
    R_next = 2 * R
    base = [_rand(g, r, H) for r in ROWS]
    resid = [_rand(g, r, H) for r in ROWS]
    B = [_rand(g, H, R, std=0.02) for _ in ROWS]
    A_next = [_rand(g, H, R_next, std=0.02) for _ in ROWS]
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(BF)
    ws_in = torch.randn(total * SPLITS_IN * R, generator=g) * 0.5
    s = 2.0
    splits_out = int(lib.swl_fused_norm_splits(R))
    # device copies stay bound to names until the kernel has run
    base_d, B_d, A_d = [b.to(cuda) for b in base], [b.to(cuda) for b in B], [a.to(cuda) for a in A_next]
    ws_in_d, w_d = ws_in.to(cuda), w.to(cuda)
    h_d = [x.to(cuda) for x in resid]
    x_d = [torch.empty(r, H, dtype=BF, device=cuda) for r in ROWS]
    ws_next = torch.zeros(total * splits_out * R_next, device=cuda)
    native.check(lib.swl_fused_resid_norm_shrink(
        n, native.i32_array(ROWS), _ptrs(native, base_d), H, _ptrs(native, B_d), R, s, ws_in_d.data_ptr(),
        SPLITS_IN, 1, _ptrs(native, h_d), H, w_d.data_ptr(), H, 1e-5, _ptrs(native, x_d), H,
        _ptrs(native, A_d), R_next, ws_next.data_ptr(), None, 0, None))
    torch.cuda.synchronize()
    t = _t_from_partials(ws_in, R)
    ws_got = ws_next.cpu().view(total, splits_out, R_next).sum(1)
    row = 0
    for i, r in enumerate(ROWS):
        ti = t[row:row + r]
        d = ref.bf(ref.mm_bf16(ti, B[i].t()).float() * s)
        h_new = ref.add_bf16(resid[i], ref.add_bf16(base[i], d))
        x = ref.rms_norm(h_new, w)
        assert_close(h_d[i].cpu(), h_new, f"slot {i} new hidden")
        assert_close(x_d[i].cpu(), x, f"slot {i} normed row")
        want = x.float() @ A_next[i].float()
        assert torch.allclose(ws_got[row:row + r], want, rtol=2e-3, atol=2e-3 * want.abs().max().item()), \
            f"slot {i} next shrink partials"
        row += r


def test_gu_silu_shrink_ragged_rows(native, cuda):
    lib = native.lib()
    g = torch.Generator().manual_seed(22)
    n, total = len(ROWS), sum(ROWS)
    base = [_rand(g, r, 2 * I) for r in ROWS]
    B = [_rand(g, 2 * I, R, std=0.02) for _ in ROWS]
    A_next = [_rand(g, I, R, std=0.02) for _ in ROWS]
    ws_in = torch.randn(total * SPLITS_IN * 2 * R, generator=g) * 0.5
    nblk = int(lib.swl_fused_silu_splits(I))
    base_d, B_d, A_d = [b.to(cuda) for b in base], [b.to(cuda) for b in B], [a.to(cuda) for a in A_next]
    ws_in_d = ws_in.to(cuda)
    act_d = [torch.empty(r, I, dtype=BF, device=cuda) for r in ROWS]
    ws_next = torch.zeros(total * nblk * R, device=cuda)
    native.check(lib.swl_fused_gu_silu_shrink(
        n, native.i32_array(ROWS), _ptrs(native, base_d), 2 * I, _ptrs(native, B_d), R, ws_in_d.data_ptr(),
        SPLITS_IN, I, _ptrs(native, act_d), I, _ptrs(native, A_d), R, ws_next.data_ptr(), None, 0, None))
    torch.cuda.synchronize()
    t = _t_from_partials(ws_in, 2 * R)
    ws_got = ws_next.cpu().view(total, nblk, R).sum(1)
    row = 0
    for i, r in enumerate(ROWS):
        ti = t[row:row + r]
        dg = ref.mm_bf16(ti[:, :R], B[i][:I].t())
        du = ref.mm_bf16(ti[:, R:], B[i][I:].t())
        gate = ref.add_bf16(base[i][:, :I], dg)
        up = ref.add_bf16(base[i][:, I:], du)
        act = ref.silu_mul(gate, up)
        assert_close(act_d[i].cpu(), act, f"slot {i} SiLU * up")
        want = act.float() @ A_next[i].float()
        assert torch.allclose(ws_got[row:row + r], want, rtol=2e-3, atol=2e-3 * want.abs().max().item()), \
            f"slot {i} Down shrink partials"
        row += r


def test_qkv_rope_ragged_rows(native, cuda):
    lib = native.lib()
    g = torch.Generator().manual_seed(23)
    n, total = len(ROWS), sum(ROWS)
    N = (HQ + 2 * HKV) * D
    ctx = [40, 0, 17]  # cached tokens before the new rows
    page = 16
    pps = [(c + r + page - 1) // page for c, r in zip(ctx, ROWS)]
    base = [_rand(g, r, N) for r in ROWS]
    B = [_rand(g, N, R, std=0.02) for _ in ROWS]
    ws_in = torch.randn(total * SPLITS_IN * 3 * R, generator=g) * 0.5
    max_pos = max(c + r for c, r in zip(ctx, ROWS)) + 1
    cs = ref.cos_sin_cache(ref.llama3_inv_freq(D), max_pos)
    npages = sum(pps)
    perm = torch.randperm(npages, generator=g).to(torch.int32)
    tables, off = [], 0
    for p in pps:
        tables.append(perm[off:off + p].contiguous())
        off += p
    kc = _rand(g, npages, page, HKV, D)
    vc = _rand(g, npages, page, HKV, D)
    kd, vd = kc.to(cuda), vc.to(cuda)
    q_rot = torch.empty(total, HQ * D, dtype=BF, device=cuda)
    base_d, B_d, ws_in_d, cs_d = [b.to(cuda) for b in base], [b.to(cuda) for b in B], ws_in.to(cuda), cs.to(cuda)
    tables_d = [t.to(cuda) for t in tables]
    seq_d = [torch.tensor([c], dtype=torch.int32, device=cuda) for c in ctx]
    native.check(lib.swl_fused_qkv_rope(
        n, native.i32_array(ROWS), _ptrs(native, base_d), N, _ptrs(native, B_d), R, ws_in_d.data_ptr(), SPLITS_IN,
        _ptrs(native, tables_d), _ptrs(native, [kd] * n), _ptrs(native, [vd] * n), _ptrs(native, seq_d), HQ, HKV,
        D, page, cs_d.data_ptr(), q_rot.data_ptr(), None, 0, None))
    torch.cuda.synchronize()
    t = _t_from_partials(ws_in, 3 * R)
    qd, kd_c, vd_c = q_rot.cpu(), kd.cpu(), vd.cpu()
    dims = [HQ * D, HKV * D, HKV * D]
    row = 0
    for i, r in enumerate(ROWS):
        ti = t[row:row + r]
        Bq, Bk, Bv = torch.split(B[i], dims, 0)
        parts = [ref.add_bf16(p, ref.mm_bf16(ti[:, j * R:(j + 1) * R], Bb.t()))
                 for j, (p, Bb) in enumerate(zip(torch.split(base[i], dims, -1), (Bq, Bk, Bv)))]
        pos = torch.arange(ctx[i], ctx[i] + r)
        q = ref.rope_neox(parts[0], pos, cs, D)
        k = ref.rope_neox(parts[1], pos, cs, D)
        assert_close(qd[row:row + r], q, f"slot {i} rotated q")
        for j in range(r):
            p_ = ctx[i] + j
            pg = int(tables[i][p_ // page])
            assert_close(kd_c[pg, p_ % page].reshape(1, -1), k[j:j + 1], f"slot {i} row {j} K append")
            assert_close(vd_c[pg, p_ % page].reshape(1, -1), parts[2][j:j + 1], f"slot {i} row {j} V append")
        row += r
