"""The LM head's sampling rule (ext_aggregator.cpp:757-787, :821-861) as
restated in oracle.reference_math.sample_token, on the CPU: the greedy path,
the temperature as a bf16 multiply by the reciprocal, top-k keeping ties at
the k-th value, the reference's top-p cut (a token whose running probability
exceeds top_p is removed, the first always kept — unlike the shifted rule of
other libraries), and the inverse-CDF draw reproducing the softmax of the
kept tokens."""
import math

import torch

from oracle import reference_math as ref

BF = torch.bfloat16


def _logits_from_probs(probs):
    return torch.log(torch.tensor(probs, dtype=torch.float64)).to(BF)


def test_greedy_and_degenerate_filters_give_the_argmax():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(500, generator=g).to(BF)
    top = int(x.float().argmax())
    x[top] = x[top] + 1.0  # a unique maximum (bf16 rounding makes ties common)
    assert ref.sample_token(x, False, 1.0, 0, 1.0, 0.7)[0] == top
    for u in (0.0, 0.5, 0.999):
        assert ref.sample_token(x, True, 1.0, 1, 1.0, u)[0] == top      # top_k = 1
        assert ref.sample_token(x, True, 1.3, 0, 0.0, u)[0] == top      # top_p = 0 keeps the first only


def test_top_p_removes_the_token_that_crosses():
    # probabilities 0.5, 0.3, 0.2: running sums 0.5, 0.8, 1.0; with top_p 0.7
    # only the first stays (the reference compares cum > top_p unshifted)
    x = _logits_from_probs([0.2, 0.5, 0.3])
    for u in (0.0, 0.4, 0.99):
        assert ref.sample_token(x, True, 1.0, 0, 0.7, u)[0] == 1
    # with top_p 0.85 the first two stay, in proportion 0.5 : 0.3
    assert ref.sample_token(x, True, 1.0, 0, 0.85, 0.1)[0] == 1
    assert ref.sample_token(x, True, 1.0, 0, 0.85, 0.7)[0] == 2


def test_top_k_keeps_ties_at_the_threshold():
    x = torch.tensor([1.0, 3.0, 2.0, 2.0, 2.0, -1.0]).to(BF)
    # k = 2: the threshold is 2.0, held by three tokens; all of them stay
    seen = {ref.sample_token(x, True, 1.0, 2, 1.0, u / 100)[0] for u in range(100)}
    assert seen == {1, 2, 3, 4}


def test_temperature_is_a_bf16_multiply_by_the_reciprocal():
    x = torch.tensor([0.37, 1.91, -0.5]).to(BF)
    inv = torch.tensor(1.0) / torch.tensor(0.7)
    scaled = (x.float() * inv).to(BF).double()
    w = torch.exp(scaled - scaled.max())
    cdf = torch.cumsum(w / w.sum(), 0)
    for u in (0.05, 0.3, 0.6, 0.95):
        want = int(torch.searchsorted(cdf, torch.tensor([u], dtype=torch.float64), right=True)[0])
        assert ref.sample_token(x, True, 0.7, 0, 1.0, u)[0] == want
    # temperatures below 0.01 are clamped to 0.01
    assert ref.sample_token(x, True, 0.0, 0, 1.0, 0.5) == ref.sample_token(x, True, 0.01, 0, 1.0, 0.5)


def test_draw_frequencies_follow_the_kept_softmax():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(40, generator=g).to(BF)
    k, p = 10, 0.9
    n = 4000
    counts = torch.zeros(40)
    for i in range(n):
        counts[ref.sample_token(x, True, 1.0, k, p, (i + 0.5) / n)[0]] += 1
    # expected: softmax over the top-10, then the nucleus, renormalised
    xs = x.double()
    top = torch.topk(xs, k).indices
    w = torch.zeros(40, dtype=torch.float64)
    w[top] = torch.exp(xs[top] - xs.max())
    order = torch.sort(xs.masked_fill(w == 0, -math.inf), descending=True, stable=True).indices[:k]
    cum = torch.cumsum(w[order], 0) / w.sum()
    stay = cum <= p
    stay[0] = True
    keep = torch.zeros(40, dtype=torch.bool)
    keep[order[stay]] = True
    want = torch.where(keep, w, torch.zeros((), dtype=torch.float64))
    want = want / want.sum()
    assert torch.allclose(counts.double() / n, want, atol=1.5 / n + 1e-9)
