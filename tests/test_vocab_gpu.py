"""Greedy next-token pick of the LM-head op (ext_aggregator.cpp:821-874:
torch.argmax over each slot's logits) through swl_argmax_rows, against
torch.argmax on the CPU: the full Llama-3.1 vocabulary, vocabularies that
are not a multiple of the vector width, padded row strides (rows that are
not 16-byte aligned), planted ties (the lowest index wins) and rows whose
maximum sits in the last or first position."""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _pick(native, logits_dev, rows, vocab, ld):
    out = torch.full((rows,), -1, dtype=torch.int64, device=logits_dev.device)
    native.check(native.lib().swl_argmax_rows(C.c_void_p(logits_dev.data_ptr()), rows, vocab, ld,
                                               C.c_void_p(out.data_ptr()), None))
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("vocab,pad", [(128256, 0), (1001, 0), (1001, 3), (64, 5), (7, 0), (32000, 8)])
def test_argmax_rows_matches_torch(native, cuda, vocab, pad):
    rows = 28
    ld = vocab + pad
    g = torch.Generator().manual_seed(vocab + pad)
    x = torch.randn(rows, ld, generator=g).to(BF)
    # planted ties: the same maximum at two or three positions of a row
    for r in range(0, rows, 3):
        i, j = sorted(torch.randperm(vocab, generator=g)[:2].tolist())
        x[r, i] = x[r, j] = 50.0
        if r % 2 == 0 and vocab > 2:
            k = torch.randint(0, vocab, (1,), generator=g).item()
            x[r, k] = 50.0
    x[1, vocab - 1] = 60.0          # maximum at the last column
    x[2, 0] = 60.0                  # maximum at the first column
    x[4, :vocab] = -3.0             # a constant row: index 0
    want = x[:, :vocab].float().argmax(dim=1)
    got = _pick(native, x.to(cuda), rows, vocab, ld)
    assert torch.equal(got, want), (got - want).nonzero()


def test_argmax_rows_ignores_nan_and_handles_infinite_rows(native, cuda):
    vocab = 1000
    x = torch.randn(3, vocab, generator=torch.Generator().manual_seed(3)).to(BF)
    x[0, 10] = float("nan")
    x[0, 500] = 40.0
    x[1, :] = float("-inf")
    x[2, 999] = float("inf")
    got = _pick(native, x.to(cuda), 3, vocab, vocab)
    assert got.tolist() == [500, 0, 999]


def test_argmax_rows_rejects_bad_arguments(native):
    lib = native.lib()
    assert lib.swl_argmax_rows(C.c_void_p(0x1000), 1, 10, 5, C.c_void_p(0x1000), None) != 0  # ld < vocab
    assert "argmax" in native.last_error()
