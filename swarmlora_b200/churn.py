"""Adapter-pool churn on one GPU: requests arrive, take a slot of a SlotGroup,
get their adapter swapped in, prefill their prompt in chunks of rows, decode
their output and leave.

This drives the engine the way the reference's worker pool is driven under
churn (workers swap adapters on a miss: adapter_manager.py:47-280, fused LoRA
refill in model_builder.py:113-183): a synthetic trace of Poisson arrivals
with lognormal prompt / output lengths and Zipf-distributed adapter ids over
a pool of adapters of mixed ranks, an LRU cache of packed adapters on the
GPU, and a step loop that packs prefill chunks and decode rows of all active
requests into one engine step (SlotGroup.enqueue_step with per-slot rows).
A step runs only the slots that hold a request (SlotGroup.subset views);
with a group that has no subset views, slots without a request run one
throw-away row from an empty context.
"""
from __future__ import annotations

import math
from collections import OrderedDict, deque
from dataclasses import dataclass, field

import numpy as np


@dataclass
class ChurnConfig:
    pool_size: int = 500                   # adapters in the pool
    ranks: tuple = (8, 16, 32)             # drawn uniformly per adapter
    rate: float = 8.0                      # Poisson arrivals per second
    prompt_median: float = 256.0           # lognormal, clipped
    prompt_sigma: float = 1.0
    prompt_clip: tuple = (32, 2048)
    output_median: float = 128.0
    output_sigma: float = 0.8
    output_clip: tuple = (16, 512)
    zipf_s: float = 1.1                    # adapter popularity
    cache_adapters: int = 32               # packed adapters kept on the GPU
    chunk: int = 16                        # prefill rows per request per step
    max_step_rows: int = 256               # token rows of one step (one attention call)


@dataclass
class Request:
    rid: int
    arrival: float                         # seconds
    adapter: int
    prompt: int                            # tokens
    output: int                            # tokens to generate
    # progress
    prefilled: int = 0
    generated: int = 0
    start: float = -1.0                    # admitted (seconds)
    first_token: float = -1.0
    done: float = -1.0


def adapter_ranks(cfg: ChurnConfig, seed: int = 0) -> np.ndarray:
    """The rank of every adapter of the pool (seeded)."""
    rng = np.random.default_rng(seed + 17)
    return rng.choice(np.asarray(cfg.ranks), size=cfg.pool_size)


def make_trace(cfg: ChurnConfig, duration_s: float, seed: int = 0) -> list[Request]:
    """Requests arriving in [0, duration_s): exponential inter-arrival times,
    adapter ids Zipf(s) over the pool (id 0 most popular), lognormal prompt
    and output lengths clipped to their ranges. Seeded and deterministic."""
    rng = np.random.default_rng(seed)
    k = np.arange(1, cfg.pool_size + 1, dtype=np.float64)
    pz = k ** (-cfg.zipf_s)
    pz /= pz.sum()
    out, t, rid = [], 0.0, 0
    while True:
        t += rng.exponential(1.0 / cfg.rate)
        if t >= duration_s:
            break
        prompt = int(np.clip(round(cfg.prompt_median * math.exp(cfg.prompt_sigma * rng.standard_normal())),
                             *cfg.prompt_clip))
        output = int(np.clip(round(cfg.output_median * math.exp(cfg.output_sigma * rng.standard_normal())),
                             *cfg.output_clip))
        out.append(Request(rid, t, int(rng.choice(cfg.pool_size, p=pz)), prompt, output))
        rid += 1
    return out


class AdapterCache:
    """LRU set of adapter ids resident on the GPU (packed, ready to copy into
    a slot). get() reports a hit, or a miss and the id it evicted."""

    def __init__(self, capacity: int):
        if capacity < 1:
            raise ValueError("the adapter cache needs room for one adapter")
        self.capacity = int(capacity)
        self._lru: OrderedDict[int, object] = OrderedDict()
        self.hits = self.misses = 0

    def get(self, aid: int, load):
        """The cached value for `aid`; on a miss calls load(aid) and may evict
        the least recently used entry. Returns (value, hit, evicted_id)."""
        if aid in self._lru:
            self._lru.move_to_end(aid)
            self.hits += 1
            return self._lru[aid], True, None
        self.misses += 1
        evicted = None
        if len(self._lru) >= self.capacity:
            evicted, _ = self._lru.popitem(last=False)
        value = load(aid)
        self._lru[aid] = value
        return value, False, evicted

    def __contains__(self, aid):
        return aid in self._lru

    def __len__(self):
        return len(self._lru)


@dataclass
class ChurnStats:
    steps: int = 0
    device_s: float = 0.0                  # sum of the measured step times
    swap_s: float = 0.0                    # device time of the admissions (loads, swaps, resets)
    load_s: float = 0.0                    # part of swap_s spent loading missed adapters
    completed: int = 0
    decode_tokens: int = 0
    prefill_tokens: int = 0
    swaps: int = 0
    cache_hits: int = 0
    cache_misses: int = 0
    ttft: list = field(default_factory=list)   # seconds, admitted requests
    tpot: list = field(default_factory=list)   # seconds per output token after the first

    def summary(self) -> dict:
        def pct(xs, q):
            return float(np.percentile(xs, q)) if xs else None
        return {"steps": self.steps, "device_s": round(self.device_s, 4), "swap_s": round(self.swap_s, 4),
                "load_s": round(self.load_s, 4),
                "completed": self.completed,
                "decode_tokens": self.decode_tokens, "prefill_tokens": self.prefill_tokens,
                "decode_tok_per_s": round(self.decode_tokens / self.device_s, 2) if self.device_s else None,
                "swaps": self.swaps, "cache_hits": self.cache_hits, "cache_misses": self.cache_misses,
                "ttft_p50_s": pct(self.ttft, 50), "ttft_p99_s": pct(self.ttft, 99),
                "tpot_p50_s": pct(self.tpot, 50), "tpot_p99_s": pct(self.tpot, 99)}


class ChurnRunner:
    """Runs a trace through a slot group. The clock is the device time of the
    steps (plus the swaps, which run on the same stream): requests whose
    arrival time has passed are admitted to free slots in arrival order.

    group needs: n, max_rows, max_len, set_adapter(i, adapter),
    set_context(i, length) and enqueue_step(stream, rows=..., tokens=...)
    (a None entry of tokens: that slot's one row is its last output). timer(fn) runs fn on `stream` and
    returns its device time in seconds. load_adapter(aid) returns the
    adapter of a pool id in a form set_adapter takes (SlotGroup: a
    PackedAdapter, so a swap is one device copy); the cache keeps what it
    returned. Admissions (loads on a miss, adapter swaps, context resets) run
    on the same stream and their time counts on the clock as well
    (stats.swap_s, of which stats.load_s loads)."""

    def __init__(self, group, trace: list[Request], cfg: ChurnConfig, load_adapter, timer, vocab: int,
                 stream=None, seed: int = 0, max_views: int = 8, capture_after: int = 8):
        self.g = group
        self.views = OrderedDict()  # active slot tuple -> subset view (LRU)
        self.max_views = int(max_views)
        self.capture_after = int(capture_after)  # all-decode steps of one busy set before its graph
        self._last_active = None
        self._repeat = 0
        self.use_views = hasattr(group, "subset")
        self.stream = stream
        self.trace = sorted(trace, key=lambda r: r.arrival)
        self.cfg = cfg
        self.cache = AdapterCache(cfg.cache_adapters)
        self.load_adapter = load_adapter
        self.timer = timer
        self.vocab = int(vocab)
        self.rng = np.random.default_rng(seed + 5)
        self.slot_req: list[Request | None] = [None] * group.n
        self.slot_adapter: list[int | None] = [None] * group.n
        self.stats = ChurnStats()

    def _admit(self, now: float, queue: deque) -> None:
        for i in range(self.g.n):
            if not queue:
                return
            if self.slot_req[i] is not None:
                continue
            req = queue.popleft()
            if req.prompt + req.output > self.g.max_len:
                raise ValueError(f"request {req.rid}: {req.prompt + req.output} tokens exceed the "
                                 f"group's context {self.g.max_len}")
            adapter, hit, _ = self.cache.get(req.adapter, self._load)
            if self.slot_adapter[i] != req.adapter:
                self.g.set_adapter(i, adapter)
                self.slot_adapter[i] = req.adapter
                self.stats.swaps += 1
            self.stats.cache_hits, self.stats.cache_misses = self.cache.hits, self.cache.misses
            self.g.set_context(i, 0)
            req.start = now
            self.slot_req[i] = req

    def _load(self, aid: int):
        out = []
        self.stats.load_s += self.timer(lambda: out.append(self.load_adapter(aid)))
        return out[0]

    def run(self, max_steps: int | None = None) -> ChurnStats:
        queue, pending = deque(), deque(self.trace)
        now = 0.0
        chunk = min(self.cfg.chunk, self.g.max_rows)
        while pending or queue or any(r is not None for r in self.slot_req):
            if max_steps is not None and self.stats.steps >= max_steps:
                break
            while pending and pending[0].arrival <= now:
                queue.append(pending.popleft())
            if queue and any(r is None for r in self.slot_req):
                dt = self.timer(lambda: self._admit(now, queue))
                now += dt
                self.stats.swap_s += dt
            if all(r is None for r in self.slot_req):
                now = pending[0].arrival  # idle until the next arrival
                continue
            rows, toks = [], []
            busy = sum(r is not None for r in self.slot_req) if self.use_views else self.g.n
            budget = self.cfg.max_step_rows - busy  # every stepped slot has one row; prefill chunks share the rest
            for i, req in enumerate(self.slot_req):
                if req is None:
                    if not self.use_views:
                        self.g.set_context(i, 0)  # a throw-away row from an empty context
                    rows.append(1)
                    toks.append([0])
                elif req.prefilled < req.prompt:
                    r = max(1, min(chunk, req.prompt - req.prefilled, 1 + budget))
                    budget -= r - 1
                    rows.append(r)
                    toks.append(self.rng.integers(0, self.vocab, size=r).tolist())
                else:
                    rows.append(1)
                    toks.append(None)  # decode: the slot's previous output token
            dt = self.timer(lambda: self._step(rows, toks))
            now += dt
            self.stats.steps += 1
            self.stats.device_s += dt
            for i, req in enumerate(self.slot_req):
                if req is None:
                    continue
                if req.prefilled < req.prompt:
                    req.prefilled += rows[i]
                    self.stats.prefill_tokens += rows[i]
                    if req.prefilled == req.prompt:  # the last prefill row yields the first token
                        req.generated, req.first_token = 1, now
                        self.stats.ttft.append(now - req.arrival)
                else:
                    req.generated += 1
                    self.stats.decode_tokens += 1
                if req.generated >= req.output and req.first_token >= 0:
                    req.done = now
                    if req.output > 1:
                        self.stats.tpot.append((req.done - req.first_token) / (req.output - 1))
                    self.stats.completed += 1
                    self.slot_req[i] = None
        return self.stats

    def _view(self, active: tuple):
        v = self.views.get(active)
        if v is None:
            v = self.views[active] = self.g.subset(active)
            while len(self.views) > self.max_views:
                _, old = self.views.popitem(last=False)
                old.close()
        else:
            self.views.move_to_end(active)
        return v

    def _step(self, rows, toks):
        """One engine step; decode rows take each slot's last output token.
        With subset views only the busy slots run: an all-decode step replays
        the view's graph, captured once the same busy set has decoded
        `capture_after` steps in a row (a capture costs about as much host
        time as a few eager steps); other steps launch eagerly. Without views, a step of
        one row per slot (decode and idle slots only) replays the group's
        captured step graph when it has one."""
        if self.use_views:
            active = tuple(i for i, r in enumerate(self.slot_req) if r is not None)
            v = self._view(active)
            rows = [rows[i] for i in active]
            toks = [toks[i] for i in active]
            if all(x == 1 for x in rows) and all(t is None for t in toks):
                self._repeat = self._repeat + 1 if active == self._last_active else 1
                self._last_active = active
                if v.graph is None and self._repeat >= self.capture_after:
                    v.capture(self.stream)
                if v.graph is not None:
                    v.replay()
                else:
                    v.enqueue_step(self.stream)
            else:
                self._last_active, self._repeat = None, 0
                v.enqueue_step(self.stream, rows=rows, tokens=toks)
            return
        if all(x == 1 for x in rows) and all(t is None or t == [0] for t in toks):
            if getattr(self.g, "graph", None) is not None:
                self.g.replay()
            else:
                self.g.enqueue_step(self.stream)
            return
        self.g.enqueue_step(self.stream, rows=rows, tokens=toks)  # None: the slot's last output, on the device
