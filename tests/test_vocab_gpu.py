"""Next-token pick of the LM-head op. Greedy (ext_aggregator.cpp:821-874:
torch.argmax over each slot's logits) through swl_argmax_rows, against
torch.argmax on the CPU: the full Llama-3.1 vocabulary, vocabularies that
are not a multiple of the vector width, padded row strides (rows that are
not 16-byte aligned), planted ties (the lowest index wins) and rows whose
maximum sits in the last or first position. Sampling (temperature, top-k,
top-p; ext_aggregator.cpp:757-787) through swl_sample_rows against the CPU
restatement in oracle.reference_math, and through the aggregator's LM-head
round with per-worker sampling states."""
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


# (do_sample, temperature, top_k, top_p) per row, cycled
SAMPLE_CASES = [(0, 1.0, 0, 1.0), (1, 1.0, 0, 1.0), (1, 0.7, 50, 1.0), (1, 1.3, 50, 0.9), (1, 1.0, 0, 0.9),
                (1, 1.0, 1, 1.0), (1, 0.5, 5, 0.5), (1, 1.0, 1000, 0.95), (1, 2.0, 0, 0.3), (1, 0.005, 0, 1.0),
                (1, 1.0, 40, 0.0)]


@pytest.mark.parametrize("vocab", [128256, 32000, 1001, 7])
def test_sampled_tokens_follow_the_reference_rule(native, cuda, vocab):
    """swl_sample_rows against oracle.reference_math: greedy rows give the
    argmax; a sampling row's token lies in the kept set (top-k with ties, the
    reference's top-p cut) and the uniform u lies in its interval of the
    kept softmax's CDF, up to the fp32 rounding of the kernel's sums. Rows
    with planted ties at the top, a constant row and rows of coarse values
    (ties everywhere, signed zeros) are included."""
    from oracle import reference_math as ref
    from swarmlora_b200.rounds import next_tokens
    rows = 2 * len(SAMPLE_CASES)
    g = torch.Generator().manual_seed(vocab)
    x = (torch.randn(rows, vocab, generator=g) * 2.0).to(BF)
    x[3, : min(4, vocab)] = 9.0          # four tied maxima
    x[7, :] = 0.5                        # all equal
    x[14, vocab // 2:] = -float("inf")   # half the vocabulary impossible
    # coarse values: many ties, +0 and -0 among them (equal, as torch compares)
    x[15:] = ((x[15:].float() * 4).round() / 4).to(BF)
    x[16:, 1::2] = torch.where(x[16:, 1::2] == 0, torch.tensor(-0.0), x[16:, 1::2].float()).to(BF)
    params = [SAMPLE_CASES[r % len(SAMPLE_CASES)] for r in range(rows)]
    u = torch.rand(rows, generator=g)
    got = next_tokens(x.to(cuda), params, u=u.to(cuda)).cpu()
    for r in range(rows):
        d, T, k, p = params[r]
        t = int(got[r])
        assert 0 <= t < vocab, (r, t)
        if not d:
            assert t == int(x[r].float().argmax()), f"row {r}: greedy {t}"
            continue
        probs, _ = ref.sample_distribution(x[r], T, k, p)
        allowed = ref.sample_allowed(x[r], T, k, p, slack=1e-5)
        assert allowed[t], f"row {r} {params[r]}: token {t} outside the kept set"
        cdf = torch.cumsum(probs, 0)
        lo, hi, ur = float(cdf[t] - probs[t]), float(cdf[t]), float(u[r])
        assert lo - 1e-4 <= ur <= hi + 1e-4, f"row {r} {params[r]}: u={ur} outside [{lo}, {hi}] of token {t}"


def test_sampling_without_uniforms_is_seeded(native, cuda):
    """With u = NULL the draws are a function of (seed, offset, row): the
    same triple repeats the tokens, another offset changes them."""
    from swarmlora_b200.rounds import next_tokens
    g = torch.Generator().manual_seed(2)
    x = torch.randn(64, 4096, generator=g).to(BF).to(cuda)
    params = [(1, 1.0, 0, 1.0)] * 64
    a = next_tokens(x, params, seed=7, offset=3).cpu()
    b = next_tokens(x, params, seed=7, offset=3).cpu()
    c = next_tokens(x, params, seed=7, offset=4).cpu()
    assert torch.equal(a, b)
    assert (a != c).sum() > 32


def test_lm_head_round_samples_with_each_workers_state(native, cuda):
    """The aggregator's LM-head round: a slot whose worker has a sampling
    state draws with it (top_k = 1 keeps only the maximum: the greedy token),
    slots without one stay greedy, and one seed repeats its draws."""
    import ctypes as C
    from swarmlora_b200 import ext_aggregator as agg
    from swarmlora_b200._native import check, i64_array, lib, ptr_array
    H, I, V, n = 256, 512, 4096, 4
    workers = [11, 12, 13, 14]
    g = torch.Generator(device=cuda).manual_seed(4)

    def w(*shape):
        return (torch.randn(*shape, generator=g, device=cuda) * 0.02).to(BF)

    def copy(dst, src, nbytes):
        check(lib().swl_copy_rows(1, ptr_array([src]), ptr_array([dst]), i64_array([nbytes]), None))
        torch.cuda.synchronize()
    lm = w(V, H)
    keep = [w(H, H), w(128, H), w(128, H), w(H, H), w(I, H), w(I, H), w(H, I), w(V, H)]
    agg.init_slot_pool(n, 0, H, I, 2, 64, 16, 2)
    try:
        agg.init_aggregator_begin(1, 0)
        agg.init_aggregator_layer(0, keep[0], keep[1], keep[2], keep[3], torch.empty(0), keep[4], keep[5], keep[6],
                                  torch.empty(0))
        agg.init_aggregator_finalize()
        agg.init_embed_lm_head_weights(keep[7], lm)
        sids = [agg.claim_slot(wid)["slot_id"] for wid in workers]
        bufs = [agg.slot_buffers(s) for s in sids]
        # slot i's hidden row points at vocabulary entry 100 + i: a unique, wide maximum
        rows = (lm[[100, 101, 102, 103]].float() * 60).to(BF)
        for i in range(n):
            copy(bufs[i][0], rows[i].data_ptr(), H * 2)

        def lm_round():
            agg.execute_round(agg.OP_LM_HEAD, 0, sids, workers, [1] * n, [1] * n)
            torch.cuda.synchronize()
            out = torch.empty(n, dtype=torch.int64, device=cuda)
            for i in range(n):
                copy(out[i].data_ptr(), bufs[i][1], 8)
            return out.cpu().tolist()
        greedy = lm_round()
        assert greedy == [100, 101, 102, 103]
        agg.set_worker_sampling(12, True, 1.0, 1, 1.0)
        assert lm_round() == greedy
        agg.set_worker_sampling(13, True, 1.0, 0, 1.0)  # the full softmax
        agg.set_sampling_seed(5)
        a = lm_round()
        agg.set_sampling_seed(5)
        b = lm_round()
        assert a == b and a[0] == 100 and a[1] == 101 and a[3] == 103 and 0 <= a[2] < V
        for wid in workers:
            agg.set_worker_sampling(wid, False)
        for s, wid in zip(sids, workers):
            agg.release_slot(s, wid)
    finally:
        agg.cleanup_slot_pool()
