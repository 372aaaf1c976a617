"""Slot-round kernel (gather -> base GEMM -> scatter) against the CPU oracle.

Covers the four per-layer rounds at the Llama-3.1-8B shapes with decode
slots (one token each), ragged per-slot token counts including empty slots
and multi-chunk M, explicit K-split (cluster) factors, bias, and the CUDA-core
cross-check kernel. Inputs are seeded; W ~ N(0, 0.02), x ~ N(0, 1).
"""
import pytest
import torch

from oracle import reference_math as ref
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu

H, I, QKV, GU = 4096, 14336, 6144, 28672
SHAPES = {"qkv": (QKV, H), "o": (H, H), "gate_up": (GU, H), "down": (H, I)}


def _case(N, K, rows, seed, with_bias=False):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    xs = [torch.randn(r, K, generator=g).to(torch.bfloat16) for r in rows]
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16) if with_bias else None
    return W, xs, b


def _run(W, xs, b, algo, splits=0, pad_rows=16):
    from swarmlora_b200.rounds import slot_gemm, device_error
    dev = torch.device("cuda:0")
    Wd = W.to(dev)
    N, K = W.shape
    # Each slot gets its own allocation sized like a pool slot (pad_rows rows),
    # so reads/writes past a slot's rows would show up as corruption.
    ins, outs = [], []
    for x in xs:
        buf = torch.zeros(max(pad_rows, x.shape[0]), K, dtype=torch.bfloat16, device=dev)
        buf[: x.shape[0]] = x.to(dev)
        ins.append(buf[: x.shape[0]])
        outs.append(torch.full((max(pad_rows, x.shape[0]), N), 7.0, dtype=torch.bfloat16, device=dev))
    slot_gemm(Wd, ins, outs, bias=b.to(dev) if b is not None else None, algo=algo, splits=splits)
    torch.cuda.synchronize()
    assert device_error() == 0
    return [o.cpu() for o in outs]


def _check(W, xs, b, outs, what):
    want = ref.slot_round(xs, W, b)
    for i, (o, w) in enumerate(zip(outs, want)):
        r = w.shape[0]
        assert_close(o[:r], w, f"{what} slot {i}")
        # rows past the slot's token count must be untouched
        assert (o[r:] == 7.0).all(), f"{what} slot {i}: wrote past its rows"


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("algo", [1, 2, 3])
def test_decode_round_28_slots(native, cuda, name, algo):
    N, K = SHAPES[name]
    W, xs, b = _case(N, K, [1] * 28, seed=100 + len(name))
    outs = _run(W, xs, b, algo)
    _check(W, xs, b, outs, f"{name}/algo{algo}")


@pytest.mark.parametrize("rows", [[1], [3, 0, 16, 1, 7], [16] * 4 + [1] * 24,
                                  [16] * 8 + [1] * 40, [64, 64, 64, 64, 44, 1],
                                  [1] * 128])  # the slot table's maximum
def test_ragged_rows(native, cuda, rows):
    N, K = 4096, 4096
    W, xs, b = _case(N, K, rows, seed=sum(rows))
    outs = _run(W, xs, b, algo=1, pad_rows=max(16, max(rows)))
    _check(W, xs, b, outs, f"rows={rows}")


@pytest.mark.parametrize("rows", [[1], [3, 0, 16, 1, 7], [1] * 64, [16, 16, 16, 15]])
def test_stream_k_ragged_and_repeatable(native, cuda, rows):
    """Stream-K rounds (<= 64 rows): ragged slots, and bit-identical results over
    repeated launches (the per-tile arrival counters reset themselves)."""
    for (N, K) in [(4096, 14336), (28672, 4096), (128256 // 4, 4096)]:
        W, xs, b = _case(N, K, rows, seed=N + sum(rows))
        outs = _run(W, xs, b, algo=3, pad_rows=max(16, max(rows)))
        _check(W, xs, b, outs, f"stream-K N={N} K={K} rows={rows}")
        again = _run(W, xs, b, algo=3, pad_rows=max(16, max(rows)))
        for o, a in zip(outs, again):
            assert torch.equal(o, a), "stream-K round is not deterministic"


@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8])
def test_explicit_splits(native, cuda, splits):
    N, K = QKV, H
    W, xs, b = _case(N, K, [1] * 28, seed=7)
    outs = _run(W, xs, b, algo=1, splits=splits)
    _check(W, xs, b, outs, f"splits={splits}")


@pytest.mark.parametrize("name,rows,splits", [("o", [1] * 28, 8), ("down", [1] * 28, 0), ("qkv", [1] * 88, 0),
                                               ("o", [2, 1, 5, 0, 9], 3), ("down", [1] * 28, 5)])
def test_global_split_matches_cluster_split(native, cuda, name, rows, splits):
    """Split-K reduced through the global-memory workspace (tuning flag) and
    across a thread-block cluster (the default) give bit-identical outputs (both sum
    the splits' fp32 partials in split order), and repeated launches agree
    (the per-tile arrival counters reset themselves); both against the
    oracle."""
    from swarmlora_b200._native import check, lib
    N, K = SHAPES[name]
    W, xs, b = _case(N, K, rows, seed=N + len(rows) + splits)
    try:
        cluster = _run(W, xs, b, algo=1, splits=splits)
        check(lib().swl_round_tune(32, 0, 0, 2))  # flags are global; the tile stays the default
        glob = _run(W, xs, b, algo=1, splits=splits)
        again = _run(W, xs, b, algo=1, splits=splits)
    finally:
        check(lib().swl_round_tune(32, 0, 0, 0))
    _check(W, xs, b, glob, f"{name} rows={len(rows)} global split-K")
    for i, (c, g2, a) in enumerate(zip(cluster, glob, again)):
        assert torch.equal(c, g2), f"slot {i}: global split-K differs from the cluster reduction"
        assert torch.equal(g2, a), f"slot {i}: global split-K is not repeatable"


@pytest.mark.parametrize("name,rows", [("gate_up", [1] * 88), ("down", [16] * 8), ("o", [16] * 12 + [1] * 20),
                                       ("qkv", [2, 0, 7] + [16] * 14), ("o", [1] * 28)])
def test_staged_token_tiles_match_gathered(native, cuda, name, rows):
    """Token tiles loaded by TMA from a packed staging copy (the default above
    128 rows) and gathered row by row from the slot buffers give
    bit-identical outputs, for every row class; against the oracle too."""
    from swarmlora_b200._native import check, lib
    N, K = SHAPES[name]
    W, xs, b = _case(N, K, rows, seed=N + sum(rows))
    m = sum(rows)
    cls = next((c for c in (32, 64, 96, 128) if m <= c), 0)
    tile = {32: (32, 4), 64: (64, 4), 96: (96, 3), 128: (128, 3), 0: (256, 3)}[cls]
    pad = max(16, max(rows))
    try:
        check(lib().swl_round_tune(cls, tile[0], tile[1], 0))
        gathered = _run(W, xs, b, algo=1, pad_rows=pad)
        check(lib().swl_round_tune(cls, tile[0], tile[1], 8))
        staged = _run(W, xs, b, algo=1, pad_rows=pad)
    finally:
        check(lib().swl_round_tune(cls, 0, 0, 0))
    _check(W, xs, b, staged, f"{name} rows={m} staged")
    for i, (g2, s2) in enumerate(zip(gathered, staged)):
        assert torch.equal(g2, s2), f"slot {i}: staged token tiles differ from gathered ones"


def test_bias_and_down_shape_ragged(native, cuda):
    W, xs, b = _case(H, I, [2, 1, 5], seed=11, with_bias=True)
    outs = _run(W, xs, b, algo=1)
    _check(W, xs, b, outs, "down+bias")


def test_rejects_bad_arguments(native, cuda):
    from swarmlora_b200.rounds import slot_gemm
    dev = torch.device("cuda:0")
    W = torch.zeros(100, 64, dtype=torch.bfloat16, device=dev)  # N not a multiple of 8
    x = torch.zeros(1, 64, dtype=torch.bfloat16, device=dev)
    y = torch.zeros(1, 100, dtype=torch.bfloat16, device=dev)
    with pytest.raises(RuntimeError, match="multiples of 8"):
        slot_gemm(W, [x], [y])
