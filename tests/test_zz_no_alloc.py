"""swl_paged_attention_noalloc: attention whose partial results live in the
library's static per-device array instead of caller scratch.

Called through the C ABI (ctypes) and compared bit for bit with
swl_paged_attention given its own scratch, on two calls in a row of different
shapes, so the second call runs over whatever the first left in the shared
array. This file is named to be collected last: it must pass both alone in a
fresh process and after every other test has used the device.
"""
import ctypes as C
import math

import pytest
import torch

BF = torch.bfloat16
HQ, HKV, D, PAGE = 32, 8, 128, 16
SCRATCH_FLOATS = 1 << 20  # SWL_NOALLOC_ATTN_SCRATCH_FLOATS


def _case(ctx, rows, seed, dev):
    g = torch.Generator().manual_seed(seed)
    n = len(ctx)
    max_len = max(c + r for c, r in zip(ctx, rows))
    pages_per = (max_len + PAGE - 1) // PAGE + 1
    num_pages = n * pages_per
    perm = torch.randperm(num_pages, generator=g).tolist()
    # the new tokens' K/V are already in the cache (as after rope_append)
    kc = torch.randn(num_pages, PAGE, HKV, D, generator=g).to(BF).to(dev)
    vc = torch.randn(num_pages, PAGE, HKV, D, generator=g).to(BF).to(dev)
    tables = [torch.tensor(perm[i * pages_per:(i + 1) * pages_per], dtype=torch.int32, device=dev)
              for i in range(n)]
    seqlens = [torch.tensor([c], dtype=torch.int32, device=dev) for c in ctx]
    q_rot = torch.randn(sum(rows), HQ * D, generator=g).to(BF).to(dev)
    return dict(rows=rows, tables=tables, kc=kc, vc=vc, seqlens=seqlens, q_rot=q_rot,
                max_len=max_len, n=n)


def _args(native, c, outs):
    n = c["n"]
    return [n, native.i32_array(c["rows"]),
            native.ptr_array([t.data_ptr() for t in c["tables"]]),
            native.ptr_array([c["kc"].data_ptr()] * n), native.ptr_array([c["vc"].data_ptr()] * n),
            native.ptr_array([s.data_ptr() for s in c["seqlens"]]),
            native.ptr_array([o.data_ptr() for o in outs]), HQ * D, HQ, HKV, D, PAGE,
            1.0 / math.sqrt(D), c["max_len"], c["q_rot"].data_ptr()]


@pytest.mark.gpu
def test_noalloc_attention_matches_scratch_entry_point(native, cuda):
    lib = native.lib()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [([1000, 3, 513, 77], [1, 1, 1, 1], 11),        # many context splits
             ([0, 40, 7, 300, 1000, 16], [16, 1, 1, 4, 1, 2], 12)]  # ragged rows, other chunk count
    for ctx, rows, seed in cases:
        c = _case(ctx, rows, seed, cuda)
        total = sum(rows)
        need = lib.swl_attention_part_floats(total, HQ, HKV, c["max_len"])
        assert 0 < need <= SCRATCH_FLOATS
        part = torch.empty(need, dtype=torch.float32, device=cuda)
        want = [torch.empty(r, HQ * D, dtype=BF, device=cuda) for r in rows]
        got = [torch.full((r, HQ * D), float("nan"), dtype=BF, device=cuda) for r in rows]
        a = _args(native, c, want)
        native.check(lib.swl_paged_attention(*a, part.data_ptr(), stream))
        native.check(lib.swl_paged_attention_noalloc(*_args(native, c, got), stream))
        torch.cuda.synchronize()
        for i, (w, o) in enumerate(zip(want, got)):
            assert torch.isfinite(w.float()).all()
            assert torch.equal(w, o), f"ctx {ctx} slot {i}: no-alloc attention differs"


def test_noalloc_attention_rejects_oversize_launch(native):
    """A shape whose partials exceed the static array fails before any CUDA
    call (so this runs without a GPU; the pointers are never dereferenced)."""
    lib = native.lib()
    hq, hkv, n, r, max_len = 8, 1, 16, 8, 4096
    total = n * r
    assert lib.swl_attention_part_floats(total, hq, hkv, max_len) > SCRATCH_FLOATS
    fake = native.ptr_array([0x1000] * n)
    st = lib.swl_paged_attention_noalloc(n, native.i32_array([r] * n), fake, fake, fake, fake, fake,
                                         hq * D, hq, hkv, D, PAGE, 0.1, max_len, C.c_void_p(0x1000),
                                         None)
    assert st != 0
    assert "static scratch holds 1048576" in native.last_error()
    # a non-positive head count is refused before the scratch size is computed
    for bad_hq in (0, -8):
        st = lib.swl_paged_attention_noalloc(n, native.i32_array([r] * n), fake, fake, fake, fake, fake,
                                             hq * D, bad_hq, hkv, D, PAGE, 0.1, 64, C.c_void_p(0x1000),
                                             None)
        assert st != 0
        assert "hq and hkv must be positive" in native.last_error()
