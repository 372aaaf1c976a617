"""The adapter-churn driver (swarmlora_b200.churn) on the CPU: the synthetic
trace's distributions, the LRU adapter cache, a full run of the step loop
against a fake slot group that records what each step asked for, and the
packed-adapter slab a swap copies."""
import numpy as np
import pytest
import torch

from swarmlora_b200 import worker_ops as wo
from swarmlora_b200.churn import AdapterCache, ChurnConfig, ChurnRunner, adapter_ranks, make_trace


def test_trace_follows_its_distributions():
    cfg = ChurnConfig()
    tr = make_trace(cfg, 300.0, seed=1)
    assert tr == make_trace(cfg, 300.0, seed=1)  # seeded
    arr = np.array([r.arrival for r in tr])
    assert np.all(np.diff(arr) >= 0) and arr[-1] < 300.0
    assert abs(len(tr) / 300.0 - cfg.rate) < 0.5  # Poisson rate
    prompts = np.array([r.prompt for r in tr])
    outputs = np.array([r.output for r in tr])
    assert prompts.min() >= 32 and prompts.max() <= 2048
    assert outputs.min() >= 16 and outputs.max() <= 512
    assert 200 <= np.median(prompts) <= 320 and 100 <= np.median(outputs) <= 160
    counts = np.bincount([r.adapter for r in tr], minlength=cfg.pool_size)
    assert counts.argmax() == 0 and counts[0] > counts[10] > 0  # Zipf: id 0 most popular
    ranks = adapter_ranks(cfg)
    assert set(np.unique(ranks)) == {8, 16, 32} and len(ranks) == cfg.pool_size


def test_adapter_cache_is_lru():
    c = AdapterCache(2)
    loads = []

    def load(aid):
        loads.append(aid)
        return f"A{aid}"
    assert c.get(1, load) == ("A1", False, None)
    assert c.get(2, load) == ("A2", False, None)
    assert c.get(1, load) == ("A1", True, None)
    assert c.get(3, load) == ("A3", False, 2)  # 2 was least recently used
    assert c.get(2, load) == ("A2", False, 1)
    assert loads == [1, 2, 3, 2] and (c.hits, c.misses) == (1, 4) and len(c) == 2


class FakeGroup:
    """Records the steps; each step's next token is a function of its inputs.
    With views=True it offers subset views (SlotGroup.subset) whose steps run
    only their slots."""

    def __init__(self, n, vocab=1000, views=False):
        self.n, self.max_rows, self.max_len, self.vocab = n, 16, 4096, vocab
        self.tokens = torch.zeros(n, dtype=torch.int64)
        self.ctx = [0] * n
        self.adapter = [None] * n
        self.steps = []   # (active slots, rows, token lists, contexts before, adapters)
        self.captures = 0
        if views:
            self.subset = lambda active: FakeView(self, active)

    def set_adapter(self, i, a):
        self.adapter[i] = a

    def set_context(self, i, length):
        self.ctx[i] = length

    def _do(self, active, rows, tokens):
        rows = rows or [1] * len(active)
        tokens = tokens or [None] * len(active)
        assert len(rows) == len(tokens) == len(active)
        assert all(t is not None or r == 1 for t, r in zip(tokens, rows))
        tokens = [[int(self.tokens[i])] if t is None else t for i, t in zip(active, tokens)]
        self.steps.append((list(active), list(rows), [list(t) for t in tokens],
                           [self.ctx[i] for i in active], [self.adapter[i] for i in active]))
        for j, i in enumerate(active):
            self.ctx[i] += rows[j]
            self.tokens[i] = (sum(tokens[j]) + 7 * i) % self.vocab

    def enqueue_step(self, stream, rows=None, tokens=None):
        self._do(list(range(self.n)), rows, tokens)


class FakeView:
    def __init__(self, g, active):
        self.g, self.active, self.n, self.graph = g, list(active), len(active), None

    def enqueue_step(self, stream, rows=None, tokens=None):
        self.g._do(self.active, rows, tokens)

    def capture(self, stream=None):
        self.graph = "captured"
        self.g.captures += 1

    def replay(self):
        self.g._do(self.active, None, None)

    def close(self):
        self.graph = None


def _run(views):
    cfg = ChurnConfig(rate=20.0, cache_adapters=3, pool_size=20, prompt_median=40, prompt_clip=(1, 80),
                      output_median=12, output_clip=(1, 30), max_step_rows=24)
    trace = make_trace(cfg, 2.0, seed=3)
    g = FakeGroup(4, views=views)
    runner = ChurnRunner(g, trace, cfg, load_adapter=lambda aid: f"adapter{aid}", timer=lambda fn: (fn(), 0.005)[1],
                         vocab=g.vocab, capture_after=3)
    return cfg, trace, g, runner.run()


@pytest.mark.parametrize("views", [False, True])
def test_runner_serves_every_request(views):
    cfg, trace, g, st = _run(views)
    assert st.completed == len(trace)
    assert st.prefill_tokens == sum(r.prompt for r in trace)
    assert st.decode_tokens == sum(r.output - 1 for r in trace)
    assert st.cache_hits + st.cache_misses == len(trace) and st.swaps <= len(trace)
    assert abs(st.load_s - 0.005 * st.cache_misses) < 1e-9 and st.swap_s >= st.load_s
    for r in trace:  # first token after the whole prompt, done after the whole output
        assert r.start >= r.arrival and r.first_token > r.start and r.done >= r.first_token
    for active, rows, toks, ctx, adapters in g.steps:
        assert all(1 <= x <= 16 for x in rows) and [len(t) for t in toks] == rows
        assert sum(rows) <= cfg.max_step_rows
        assert all(c + x <= g.max_len for c, x in zip(ctx, rows))
        if views:  # only busy slots step, each with its request's adapter
            assert all(a is not None for a in adapters)
        else:
            assert active == list(range(g.n))
    if views:
        assert any(len(a) < g.n for a, *_ in g.steps) and g.captures > 0
        # a slot's context grows only by the rows it ran: every request's
        # prompt and output, never a throw-away row
        assert sum(sum(rows) for _, rows, *_ in g.steps) == st.prefill_tokens + st.decode_tokens
    s = st.summary()
    assert s["decode_tok_per_s"] > 0 and s["ttft_p50_s"] is not None


def _tiny_adapter(g, r, H=64, I=96, q=64, kv=32):
    dims = {"q": (H, q), "k": (H, kv), "v": (H, kv), "o": (q, H), "gate": (H, I), "up": (H, I), "down": (I, H)}
    return [{nm: ((torch.randn(r, i, generator=g) * 0.02).to(torch.bfloat16),
                  (torch.randn(o, r, generator=g) * 0.02).to(torch.bfloat16)) for nm, (i, o) in dims.items()}
            for _ in range(3)]


def test_packed_adapter_slab_layout_and_swap():
    """Adapters of ranks 8 and 16 packed at rank 16 share one slab layout;
    the slab's views hold the packed tensors, start on 512-byte boundaries,
    and copying one slab into another swaps every layer's tensors."""
    g = torch.Generator().manual_seed(4)
    R, alpha = 16, 32

    def pack(ad):
        r = int(ad[0]["q"][0].shape[0])
        layers = [wo.pack_lora_layer(w, alpha / r, pad_rank=R, post_scale=alpha / R) for w in ad]
        return layers, wo.pack_lora_slab(layers, rank=r)
    la, pa = pack(_tiny_adapter(g, 8))
    lb, pb = pack(_tiny_adapter(g, 16))
    assert pa.slab.numel() == pb.slab.numel() and (pa.rank, pb.rank) == (8, 16)
    base = pa.slab.data_ptr()
    for packed, layers in ((pa, la), (pb, lb)):
        for v, L in zip(packed.layers, layers):
            assert v.rank == R
            for f in wo.LORA_FIELDS:
                t = getattr(v, f)
                assert torch.equal(t, getattr(L, f)) and t.is_contiguous()
                assert t.untyped_storage().data_ptr() == packed.slab.untyped_storage().data_ptr()
                assert (t.data_ptr() - packed.slab.data_ptr()) % 512 == 0
    assert all((getattr(v, f).data_ptr() - base) % 512 == 0 for v in pa.layers for f in wo.LORA_FIELDS)
    pa.slab.copy_(pb.slab)  # the swap: one copy replaces every tensor
    for v, L in zip(pa.layers, lb):
        for f in wo.LORA_FIELDS:
            assert torch.equal(getattr(v, f), getattr(L, f))
