"""Whole decode steps of the slot-group engine against the CPU oracle.

Llama-3.1-8B layer shapes with 2 layers and a 4096-entry vocabulary (so the
CPU oracle runs in seconds), 5 slots with ragged KV contexts (including an
empty one and page boundaries), one slot without an adapter, 3 greedy steps
with the generated token fed back. Checks the last-layer hidden state, the
LM-head input, the greedy tokens, and that a replayed CUDA graph of the step
reproduces the eager run exactly.
"""
import copy

import pytest
import torch

from oracle.decode import decode_step
from tests.tolerances import ATOL_RMS_MULTILAYER, assert_close

pytestmark = pytest.mark.gpu
BF_ULP = 2.0 ** -7


def _cpu(x):
    if isinstance(x, torch.Tensor):
        return x.cpu()
    if isinstance(x, list):
        return [_cpu(v) for v in x]
    if isinstance(x, dict):
        return {k: _cpu(v) for k, v in x.items()}
    if isinstance(x, tuple):
        return tuple(_cpu(v) for v in x)
    if x is None:
        return None
    out = copy.copy(x)
    for k, v in vars(x).items():
        setattr(out, k, _cpu(v))
    return out


def _check_tokens(got, want, logits, what):
    for i, (g, w) in enumerate(zip(got.tolist(), want.tolist())):
        if g != w:  # tolerate a tie within one bf16 ulp of the maximum logit
            lg = logits[i].float()
            assert lg[g] >= lg.max() - BF_ULP * lg.max().abs(), f"{what}: slot {i} token {g} != {w}"


@pytest.mark.parametrize("fused", [True, False])
def test_engine_matches_oracle_and_graph_replay(native, cuda, fused):
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    ctx = [20, 0, 31, 100, 7]
    n = len(ctx)
    base = random_base(cfg, seed=1, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=10 + i, device=cuda) if i != 2 else None for i in range(n)]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=8, seed=3, fused=fused)
    try:
        base_c, ad_c = _cpu(base), _cpu(adapters)
        kc = [k.cpu() for k in grp.k_cache]
        vc = [v.cpu() for v in grp.v_cache]
        kc0 = [k.clone() for k in kc]
        vc0 = [v.clone() for v in vc]
        bts = [t.tolist() for t in grp.block_tables]
        tokens = [5, 4095, 17, 0, 1234]
        seq = list(ctx)
        grp.tokens.copy_(torch.tensor(tokens))
        eager = []
        stream = torch.cuda.current_stream()
        for step in range(3):
            grp.enqueue_step(stream)
            torch.cuda.synchronize()
            got = grp.tokens.cpu()
            want, final, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, seq, tokens)
            assert_close(grp.h, h_last, f"step {step} last-layer hidden", atol_rms=ATOL_RMS_MULTILAYER)
            assert_close(grp.read_slot_rows("in", cfg.hidden), final, f"step {step} LM-head input",
                         atol_rms=ATOL_RMS_MULTILAYER)
            _check_tokens(got, want, logits, f"step {step}")
            eager.append(got.clone())
            tokens = got.tolist()  # feed back our own tokens (the oracle follows them)
            seq = [s + 1 for s in seq]
        assert grp.seqlens.cpu().tolist() == seq
        # graph replay from the initial state reproduces the eager tokens
        for l in range(cfg.layers):
            grp.k_cache[l].copy_(kc0[l])
            grp.v_cache[l].copy_(vc0[l])
        grp.reset_positions()
        grp.tokens.copy_(torch.tensor([5, 4095, 17, 0, 1234]))
        grp.capture()
        for step in range(3):
            grp.replay()
            torch.cuda.synchronize()
            assert torch.equal(grp.tokens.cpu(), eager[step]), f"graph step {step} differs"
    finally:
        grp.close()


def test_engine_pdl_matches_serialized_launches(native, cuda):
    """Programmatic dependent launch (kernels start while the previous one
    finishes) leaves every result bit-identical to fully serialized launches,
    eager and replayed from a CUDA graph."""
    import swarmlora_b200 as swl
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    ctx = [20, 0, 31, 100, 7, 250]
    base = random_base(cfg, seed=1, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=10 + i, device=cuda) if i != 2 else None for i in range(len(ctx))]
    results = {}
    for pdl in (False, True):
        prev = swl.set_pdl(pdl)
        grp = SlotGroup(cfg, base, adapters, ctx, max_new=8, seed=3)
        try:
            grp.tokens.copy_(torch.tensor([5, 4095, 17, 0, 1234, 77]))
            stream = torch.cuda.current_stream()
            grp.enqueue_step(stream)
            grp.capture()
            for _ in range(3):
                grp.replay()
            torch.cuda.synchronize()
            results[pdl] = (grp.tokens.cpu(), grp.h.cpu(), grp.read_slot_rows("in", cfg.hidden),
                            [k.cpu() for k in grp.k_cache], [v.cpu() for v in grp.v_cache])
        finally:
            swl.set_pdl(prev)
            grp.close()
    a, b = results[False], results[True]
    assert torch.equal(a[0], b[0])
    assert torch.equal(a[1], b[1])
    assert torch.equal(a[2], b[2])
    for x, y in zip(a[3] + a[4], b[3] + b[4]):
        assert torch.equal(x, y)


def test_qkv_round_with_rope_epilogue_matches_separate_launches(native, cuda):
    """The QKV round carrying the RoPE epilogue (swl_agg_execute_qkv_rope_round)
    against the round followed by swl_fused_qkv_rope: bit-identical q, K/V
    cache appends, hidden states and tokens over two steps, with ragged
    contexts (page boundaries, an empty context) and a slot without adapter."""
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    ctx = [20, 0, 31, 100, 7, 15, 16]
    base = random_base(cfg, seed=4, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=40 + i, device=cuda) if i != 3 else None for i in range(len(ctx))]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=8, seed=5)
    try:
        kc0 = [k.clone() for k in grp.k_cache]
        vc0 = [v.clone() for v in grp.v_cache]
        runs = {}
        for fused_rope in (False, True):
            for l in range(cfg.layers):
                grp.k_cache[l].copy_(kc0[l])
                grp.v_cache[l].copy_(vc0[l])
            grp.reset_positions()
            grp.tokens.copy_(torch.tensor([3, 99, 4000, 1, 2, 77, 1024]))
            grp.qkv_rope_fused = fused_rope
            out = []
            for _ in range(2):
                grp.enqueue_step(torch.cuda.current_stream())
                torch.cuda.synchronize()
                out.append((grp.tokens.cpu(), grp.h.cpu(), grp.q_rot.cpu()))
            out.append(([k.cpu() for k in grp.k_cache], [v.cpu() for v in grp.v_cache]))
            runs[fused_rope] = out
        for step in range(2):
            for a, b in zip(runs[False][step], runs[True][step]):
                assert torch.equal(a, b), f"step {step}: fused QKV/RoPE round differs"
        for a, b in zip(runs[False][2][0] + runs[False][2][1], runs[True][2][0] + runs[True][2][1]):
            assert torch.equal(a, b), "K/V caches differ"
    finally:
        grp.close()


def test_mixed_rank_adapters_and_hot_swap(native, cuda):
    """Adapters of ranks 8, 16 and 32 in one group (the churn configuration's
    rank mix), packed at the group's rank 32 with each adapter's own alpha/r
    (load_lora_fast, model_builder.py:147-149), against the CPU oracle; then
    two slots swap adapters in place (one to another rank) and both the eager
    step and the CUDA graph captured before the swap follow the oracle."""
    from oracle.decode import decode_step
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096, rank=32, alpha=32)
    ranks = [8, 16, 32, 8, 16]
    ctx = [20, 5, 31, 100, 7]
    base = random_base(cfg, seed=2, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=70 + i, device=cuda, rank=r) for i, r in enumerate(ranks)]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=8, seed=6)
    try:
        base_c = _cpu(base)
        kc = [k.cpu() for k in grp.k_cache]
        vc = [v.cpu() for v in grp.v_cache]
        kc0 = [k.clone() for k in grp.k_cache]
        vc0 = [v.clone() for v in grp.v_cache]
        bts = [t.tolist() for t in grp.block_tables]
        tokens, seq = [11, 22, 33, 44, 55], list(ctx)
        grp.tokens.copy_(torch.tensor(tokens))
        stream = torch.cuda.current_stream()

        def check_step(what, ad_c):
            nonlocal tokens, seq
            grp.enqueue_step(stream)
            torch.cuda.synchronize()
            got = grp.tokens.cpu()
            want, final, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, seq, tokens)
            assert_close(grp.h, h_last, f"{what} last-layer hidden", atol_rms=ATOL_RMS_MULTILAYER)
            _check_tokens(got, want, logits, what)
            tokens, seq = got.tolist(), [s + 1 for s in seq]
            return got

        ad_c = _cpu(adapters)
        check_step("mixed ranks step 0", ad_c)
        grp.capture()  # before the swap: the graph must pick the swapped adapters up
        check_step("mixed ranks step 1", ad_c)
        # swap slot 1 (rank 16 -> 32) and slot 3 (rank 8 -> 16)
        new1 = random_adapter(cfg, seed=91, device=cuda, rank=32)
        new3 = random_adapter(cfg, seed=93, device=cuda, rank=16)
        grp.set_adapter(1, new1)
        grp.set_adapter(3, new3)
        ad_c[1], ad_c[3] = _cpu(new1), _cpu(new3)
        eager = check_step("after swap", ad_c)
        # the graph captured before the swap, from the same state, gives the same token
        k_now = [k.clone() for k in grp.k_cache]
        v_now = [v.clone() for v in grp.v_cache]
        for l in range(cfg.layers):
            grp.k_cache[l].copy_(kc0[l])
            grp.v_cache[l].copy_(vc0[l])
        grp.reset_positions()
        grp.tokens.copy_(torch.tensor([11, 22, 33, 44, 55]))
        grp.set_adapter(1, adapters[1])  # replay the first two steps with the original adapters
        grp.set_adapter(3, adapters[3])
        for _ in range(2):
            grp.replay()
        grp.set_adapter(1, grp.pack_adapter(new1))  # packed slabs: one device copy per swap
        grp.set_adapter(3, grp.pack_adapter(new3))
        grp.replay()
        torch.cuda.synchronize()
        assert torch.equal(grp.tokens.cpu(), eager), "graph replay after the swap differs from the eager step"
        for l in range(cfg.layers):
            assert torch.equal(grp.k_cache[l], k_now[l]) and torch.equal(grp.v_cache[l], v_now[l])
    finally:
        grp.close()


def test_mixed_prefill_and_decode_step(native, cuda):
    """The mixed configuration's step through the engine: slots carrying
    prefill chunks (16, 5 and 3 new tokens, one of them into an empty
    context) next to decode rows, packed into each round's gathered rows,
    against the CPU oracle (every new row's K / V appended, attention causal
    among a slot's new rows, the next token from each slot's last row); then
    a plain decode step from the resulting state."""
    from oracle.decode import decode_step
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    ctx = [0, 20, 31, 100, 7]
    rows = [16, 1, 5, 1, 3]
    base = random_base(cfg, seed=3, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=80 + i, device=cuda) if i != 1 else None for i in range(len(ctx))]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=32, seed=8)
    try:
        base_c, ad_c = _cpu(base), _cpu(adapters)
        kc = [k.cpu() for k in grp.k_cache]
        vc = [v.cpu() for v in grp.v_cache]
        bts = [t.tolist() for t in grp.block_tables]
        g = torch.Generator().manual_seed(9)
        toks = [torch.randint(0, cfg.vocab, (r,), generator=g).tolist() for r in rows]
        stream = torch.cuda.current_stream()
        grp.enqueue_step(stream, rows=rows, tokens=toks)
        torch.cuda.synchronize()
        want, final, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, list(ctx), toks)
        got_h = torch.stack([grp.h_rows[i, r - 1] for i, r in enumerate(rows)])
        assert_close(got_h, h_last, "mixed step: last row's last-layer hidden", atol_rms=ATOL_RMS_MULTILAYER)
        got = grp.tokens.cpu()
        _check_tokens(got, want, logits, "mixed step")
        seq = [c + r for c, r in zip(ctx, rows)]
        assert grp.seqlens.cpu().tolist() == seq
        for l in range(cfg.layers):  # layer l > 0's K / V come from hidden states after l layers
            tol = {} if l == 0 else {"atol_rms": ATOL_RMS_MULTILAYER}
            assert_close(grp.k_cache[l], kc[l], f"layer {l} K cache after the mixed step", **tol)
            assert_close(grp.v_cache[l], vc[l], f"layer {l} V cache after the mixed step", **tol)
        # a plain decode step continues from there
        tokens = got.tolist()
        grp.enqueue_step(stream)
        torch.cuda.synchronize()
        want, final, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, seq, tokens)
        assert_close(grp.h, h_last, "decode after the mixed step: last-layer hidden", atol_rms=ATOL_RMS_MULTILAYER)
        _check_tokens(grp.tokens.cpu(), want, logits, "decode after the mixed step")
    finally:
        grp.close()


def test_subset_view_steps_only_its_slots(native, cuda):
    """SlotGroup.subset: a view over slots 0, 2 and 4 of a five-slot group
    runs a decode step and then a mixed step (a 6-row prefill chunk on slot
    2) for those slots only, against the CPU oracle on the same three slots;
    the idle slots' positions and pages stay untouched, and the view's
    captured graph replays its decode step bit-identically."""
    from oracle.decode import decode_step
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    ctx = [12, 40, 3, 77, 25]
    active = [0, 2, 4]
    base = random_base(cfg, seed=4, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=60 + i, device=cuda) for i in range(len(ctx))]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=16, seed=9)
    try:
        base_c = _cpu(base)
        ad_c = [_cpu(adapters[i]) for i in active]
        kc = [k.cpu() for k in grp.k_cache]
        vc = [v.cpu() for v in grp.v_cache]
        bts = [grp.block_tables[i].tolist() for i in active]
        idle_pages = [p for i in (1, 3) for p in grp.block_tables[i].tolist()]
        idle_k = [k.cpu()[idle_pages] for k in grp.k_cache]
        tokens = [101, 202, 303, 404, 505]
        grp.tokens.copy_(torch.tensor(tokens))
        view = grp.subset(active)
        stream = torch.cuda.current_stream()
        view.enqueue_step(stream)
        torch.cuda.synchronize()
        seq = [ctx[i] for i in active]
        want, final, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, seq, [tokens[i] for i in active])
        got = grp.tokens.cpu()
        assert_close(grp.h[active], h_last, "view decode: last-layer hidden", atol_rms=ATOL_RMS_MULTILAYER)
        _check_tokens(got[active], want, logits, "view decode")
        assert got[1] == 202 and got[3] == 404, "idle slots' tokens changed"
        assert grp.seqlens.cpu().tolist() == [13, 40, 4, 77, 26]
        assert all(torch.equal(k.cpu()[idle_pages], k0) for k, k0 in zip(grp.k_cache, idle_k))
        # a mixed step on the view: slot 2 prefills 6 rows, slots 0 and 4 decode
        seq = [s + 1 for s in seq]
        g = torch.Generator().manual_seed(2)
        chunk = torch.randint(0, cfg.vocab, (6,), generator=g).tolist()
        dec = got.tolist()
        view.enqueue_step(stream, rows=[1, 6, 1], tokens=[None, chunk, None])
        torch.cuda.synchronize()
        want, final, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, seq,
                                                  [[dec[0]], chunk, [dec[4]]])
        got_h = torch.stack([grp.h_rows[i, r - 1] for i, r in zip(active, [1, 6, 1])])
        assert_close(got_h, h_last, "view mixed step: last row's hidden", atol_rms=ATOL_RMS_MULTILAYER)
        _check_tokens(grp.tokens.cpu()[active], want, logits, "view mixed step")
        assert grp.seqlens.cpu().tolist() == [14, 40, 10, 77, 27]
        # the view's graph: replay from a saved state equals the eager step
        state = ([k.clone() for k in grp.k_cache], [v.clone() for v in grp.v_cache], grp.seqlens.clone(),
                 grp.tokens.clone())
        view.enqueue_step(stream)
        torch.cuda.synchronize()
        eager = (grp.tokens.clone(), [k.clone() for k in grp.k_cache], grp.seqlens.clone())
        view.capture()  # on a side stream (not the default one)
        for l in range(cfg.layers):
            grp.k_cache[l].copy_(state[0][l])
            grp.v_cache[l].copy_(state[1][l])
        grp.seqlens.copy_(state[2])
        grp.tokens.copy_(state[3])
        view.replay()
        torch.cuda.synchronize()
        assert torch.equal(grp.tokens, eager[0]) and torch.equal(grp.seqlens, eager[2])
        assert all(torch.equal(a, b) for a, b in zip(grp.k_cache, eager[1]))
        view.close()
    finally:
        grp.close()


def test_profile_step_reports_the_reference_line(native, cuda, capsys):
    """SlotGroup.profile_step: one real step with per-launch device times,
    and the `[LAYER_PROFILE]` line in the reference's key=value format
    (worker_sync.py:1774-1777), parsed the way benchmarks/ipc_overhead.py
    parses it."""
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    ctx = [5, 17, 40]
    base = random_base(cfg, seed=5, device=cuda)
    grp = SlotGroup(cfg, base, [random_adapter(cfg, seed=90 + i, device=cuda) for i in range(3)], ctx,
                    max_new=8, seed=2)
    try:
        grp.tokens.copy_(torch.tensor([1, 2, 3]))
        prof = grp.profile_step(print_line=True)
        assert grp.seqlens.cpu().tolist() == [6, 18, 41]
        kinds = ("embed", "round", "attention", "epilogue", "lm_head")
        assert all(prof[k] > 0 for k in kinds)
        assert sum(prof[k] for k in kinds) <= prof["device_us"] + 1.0 <= prof["wall_us"] + 2.0
        line = [ln for ln in capsys.readouterr().out.splitlines() if "[LAYER_PROFILE]" in ln][-1]
        parts = {}
        for tok in line.split():
            if "=" in tok:
                k, v = tok.split("=", 1)
                parts[k] = float(v)
        assert {"gather_us", "scatter_us", "compute_us", "wall_us", "ipc_pct"} <= set(parts)
        assert parts["gather_us"] == parts["scatter_us"] == 0 and parts["slots"] == 3
    finally:
        grp.close()


def test_engine_long_contexts_32_slots_match_oracle(native, cuda):
    """The long-context configuration's shape (32 slots with their own
    rank-16 adapters, contexts U[1024, 4096]) at 2 layers: two decode steps
    against the CPU oracle (last-layer hidden state, LM-head input, greedy
    tokens). Rounds of M = 32 and attention rows of 64 to 256 pages."""
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    n = 32
    g = torch.Generator().manual_seed(2024)
    ctx = [int(c) for c in torch.randint(1024, 4091, (n,), generator=g)]
    base = random_base(cfg, seed=5, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=50 + i, device=cuda) for i in range(n)]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=4, seed=9)
    try:
        base_c, ad_c = _cpu(base), _cpu(adapters)
        kc = [k.cpu() for k in grp.k_cache]
        vc = [v.cpu() for v in grp.v_cache]
        bts = [t.tolist() for t in grp.block_tables]
        tokens = torch.randint(0, cfg.vocab, (n,), generator=g).tolist()
        grp.tokens.copy_(torch.tensor(tokens))
        seq = list(ctx)
        stream = torch.cuda.current_stream()
        for step in range(2):
            grp.enqueue_step(stream)
            torch.cuda.synchronize()
            got = grp.tokens.cpu()
            want, final, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, seq, tokens)
            assert_close(grp.h, h_last, f"step {step} last-layer hidden", atol_rms=ATOL_RMS_MULTILAYER)
            assert_close(grp.read_slot_rows("in", cfg.hidden), final, f"step {step} LM-head input",
                         atol_rms=ATOL_RMS_MULTILAYER)
            _check_tokens(got, want, logits, f"step {step}")
            tokens = got.tolist()
            seq = [x + 1 for x in seq]
        assert grp.seqlens.cpu().tolist() == seq
    finally:
        grp.close()


def test_config2_full_size_step_properties(native, cuda):
    """BASELINE config 2 at its full size (32 layers, vocabulary 128256, 28
    slots with their own rank-16 adapters, contexts U[256, 1024]), checked
    through properties that hold at any size: a step writes exactly one K
    and one V row per slot and layer (at the slot's position; every other
    byte of the page pools is unchanged) and advances every position by one;
    the next tokens are valid ids; and a CUDA-graph replay from the same
    state reproduces the eager step bit for bit (tokens, hidden rows, every
    cache byte)."""
    from swarmlora_b200.engine import LLAMA_3_1_8B, SlotGroup, random_adapter, random_base
    cfg = LLAMA_3_1_8B
    n = 28
    g = torch.Generator().manual_seed(1234)
    ctx = [int(c) for c in torch.randint(256, 1025, (n,), generator=g)]
    base = random_base(cfg, seed=1, device=cuda)
    adapters = [random_adapter(cfg, seed=100 + i, device=cuda) for i in range(n)]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=4, seed=0)
    try:
        tokens0 = torch.randint(0, cfg.vocab, (n,), generator=g).to(cuda)
        grp.tokens.copy_(tokens0)
        k0 = [k.clone() for k in grp.k_cache]
        v0 = [v.clone() for v in grp.v_cache]
        stream = torch.cuda.current_stream()
        grp.enqueue_step(stream)
        torch.cuda.synchronize()
        eager = (grp.tokens.clone(), grp.h.clone())
        assert grp.seqlens.cpu().tolist() == [c + 1 for c in ctx]
        assert int(eager[0].min()) >= 0 and int(eager[0].max()) < cfg.vocab
        # exactly the (page, offset) rows at each slot's position changed
        want = {(int(grp.block_tables[i][c // cfg.page]), c % cfg.page) for i, c in enumerate(ctx)}
        for l in range(cfg.layers):
            for now, before, what in ((grp.k_cache[l], k0[l], "K"), (grp.v_cache[l], v0[l], "V")):
                rows = (now != before).flatten(2).any(-1).nonzero().tolist()
                assert {tuple(r) for r in rows} == want, f"layer {l} {what}: rows written != the new rows"
        kn = [k.clone() for k in grp.k_cache]
        vn = [v.clone() for v in grp.v_cache]
        # replay from the same starting state
        for l in range(cfg.layers):
            grp.k_cache[l].copy_(k0[l])
            grp.v_cache[l].copy_(v0[l])
        grp.reset_positions()
        grp.tokens.copy_(tokens0)
        grp.capture()
        grp.replay()
        torch.cuda.synchronize()
        assert torch.equal(grp.tokens, eager[0]) and torch.equal(grp.h, eager[1])
        assert all(torch.equal(a, b) for a, b in zip(grp.k_cache + grp.v_cache, kn + vn))
    finally:
        grp.close()


def test_mixed_step_device_tokens_and_graph_replay(native, cuda):
    """A mixed step whose one-row slots pass None (their row is the slot's
    last output, read on the device) equals the step with the ids given,
    and the same step from a CUDA graph of the row pattern (ids staged in
    tok_in) is bit-identical: tokens, hidden rows, positions and caches."""
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    ctx = [0, 20, 31, 100, 7]
    rows = [16, 1, 5, 1, 3]
    base = random_base(cfg, seed=3, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=80 + i, device=cuda) if i != 1 else None for i in range(len(ctx))]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=32, seed=8)
    try:
        g = torch.Generator().manual_seed(9)
        toks = [torch.randint(0, cfg.vocab, (r,), generator=g).tolist() for r in rows]
        stream = torch.cuda.current_stream()
        kc0 = [k.clone() for k in grp.k_cache]
        vc0 = [v.clone() for v in grp.v_cache]

        def restore():
            for l in range(cfg.layers):
                grp.k_cache[l].copy_(kc0[l])
                grp.v_cache[l].copy_(vc0[l])
            grp.reset_positions()
        grp.enqueue_step(stream, rows=rows, tokens=toks)
        torch.cuda.synchronize()
        given = (grp.tokens.clone(), grp.h_rows.clone(), [k.clone() for k in grp.k_cache],
                 [v.clone() for v in grp.v_cache], grp.seqlens.clone())

        def same(what):
            assert torch.equal(grp.tokens, given[0]) and torch.equal(grp.seqlens, given[4]), what
            assert all(torch.equal(grp.h_rows[i, :r], given[1][i, :r]) for i, r in enumerate(rows)), what
            assert all(torch.equal(a, b) for a, b in zip(grp.k_cache + grp.v_cache, given[2] + given[3])), what
        restore()
        grp.tokens.copy_(torch.tensor([t[0] for t in toks]))
        grp.enqueue_step(stream, rows=rows, tokens=[None if r == 1 else t for t, r in zip(toks, rows)])
        torch.cuda.synchronize()
        same("one-row slots' tokens read on the device")
        grp.capture(rows=rows)
        restore()
        for i, t in enumerate(toks):
            grp.tok_in[i, :len(t)].copy_(torch.tensor(t))
        grp.replay()
        torch.cuda.synchronize()
        same("graph replay of the row pattern")
    finally:
        grp.close()
