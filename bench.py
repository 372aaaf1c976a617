"""Decode benchmark of the SwarmLoRA aggregator hot path on B200.

Workload: Llama-3.1-8B architecture (32 layers, hidden
4096, 32/8 heads, intermediate 14336, vocab 128256), random-init bf16 weights
~N(0, 0.02); 28 decode slots per GPU, each with its own r=16 / alpha=32
adapter on all 7 projections (A, B ~ N(0, 0.02)); per-slot KV context
~U[256, 1024] in pages of 16; one token per slot per step (greedy).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Our arm: every GPU runs its own aggregator group (adapter workers are
partitioned per GPU, no collective on the data path). One step = one decode
token for all slots of the group, replayed from a CUDA graph of the fixed
launch sequence. `value` is device-timed (CUDA events, max over ranks);
`e2e` re-times the step through the same API with the step's input token ids
copied from pinned host memory and the next tokens read back every step.
The per-round kernel times (the metric's "us per gather-GEMM-scatter round")
and the roofline of the dominant kernel come from a second timed phase that
replays each round kind over all 32 layers' weights.

Reference arm (--impl reference): the reference path restated on the host
CPU (oracle/, torch on CPU with all host threads), bounded to one decoder
layer per step and extrapolated to the 32-layer token.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s/GPU (Llama-3.1-8B shape, N=28 slots)"
UNIT = "tok/s"
N_SLOTS = 28


def metric_for(slots: int) -> str:
    """The headline metric's name with the run's slot count (the headline
    configuration runs 28)."""
    return METRIC if slots == N_SLOTS else METRIC.replace("N=28", f"N={slots}")
CTX_LO, CTX_HI = 256, 1024
MAX_NEW = 160


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--slots", type=int, default=N_SLOTS)
    ap.add_argument("--ctx-lo", type=int, default=CTX_LO,
                    help="per-slot context ~U[lo, hi] (config 2: 256..1024; config 5: --slots 32 --ctx-lo 1024 --ctx-hi 4096)")
    ap.add_argument("--ctx-hi", type=int, default=CTX_HI)
    ap.add_argument("--layers", type=int, default=32,
                    help="decoder layers (32 = the benchmarked model; fewer only for small profiling cases)")
    ap.add_argument("--vocab", type=int, default=128256,
                    help="vocabulary (128256 = the benchmarked model; smaller only for profiling cases)")
    ap.add_argument("--checkpoint", default=None, metavar="DIR",
                    help="decode with the base weights of an HF Llama checkpoint directory instead of random ones")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-step", action="store_true",
                    help="bracket the first timed step with cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    ap.add_argument("--profile-round", choices=["qkv", "o", "gate_up", "down"], default=None,
                    help="run only --steps launches of one round kind at M=--slots (small ncu case)")
    ap.add_argument("--round-rows", type=int, default=1,
                    help="token rows per slot for --profile-round (M = slots x rows; a prefill-packed round)")
    ap.add_argument("--round-algo", type=int, default=0,
                    help="round kernel for --profile-round: 0 auto, 1 cluster split-K, 3 stream-K")
    ap.add_argument("--attn-chunk-pages", type=int, default=0, help="attention pages per chunk (0 = auto)")
    ap.add_argument("--attn-stages", type=int, default=0, help="attention page-ring depth 2..4 (0 = auto)")
    ap.add_argument("--round-flags", type=int, default=0,
                    help="round kernel flags (swl_round_tune): 1 gather spin, 2 global-memory split-K, "
                         "4 L2 prefetch of the W tiles beyond the ring")
    ap.add_argument("--round-tile", default="",
                    help="decode-class round tile as ROWSxSTAGES, e.g. 32x4 (swl_round_tune; default: automatic)")
    ap.add_argument("--attn-lane-copies", action="store_true",
                    help="attention K/V pages by per-lane cp.async copies instead of TMA")
    ap.add_argument("--attn-groups", type=int, default=0,
                    help="attention kv head groups 1/2/4/8: CTAs sharing one page's heads (0 = auto)")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch every kernel fully serialized (no programmatic dependent launch)")
    ap.add_argument("--churn", type=float, default=0.0, metavar="SECONDS",
                    help="adapter-pool churn on one GPU for SECONDS of arrivals (ranks 8/16/32, swap on miss)")
    ap.add_argument("--churn-slots", type=int, default=64)
    ap.add_argument("--churn-from-disk", action="store_true",
                    help="churn: misses read PEFT adapter files (written to a temporary pool before the run)")
    ap.add_argument("--mixed", action="store_true",
                    help="BASELINE config 3 on one GPU: prefill chunks of 4 slots packed beside 24 decode rows")
    ap.add_argument("--mixed-chunk", type=int, default=16,
                    help="prefill rows per prefill slot per step (16 = the reference's max_seq_per_step)")
    ap.add_argument("--shard", action="store_true",
                    help="column-sharded base weights over 2 GPUs (one slot group; torchrun, --gpus 2)")
    ap.add_argument("--profile-layers", type=int, default=0, metavar="N",
                    help="print N per-step [LAYER_PROFILE] lines (the reference worker's PROFILE_LAYERS format) "
                         "for the decode workload and exit")
    ap.add_argument("--protocol", default="28",
                    help="worker-client counts (comma separated) for the decode through the drop-in protocol "
                         "(aggregator main loop + native worker clients over the shared-memory ring), each "
                         "with event completion (with and without per-segment graphs) and host completion "
                         "(the reference's); 'off' skips it")
    ap.add_argument("--profile-attention", action="store_true",
                    help="run only --steps paged-attention launches over one layer's KV (small ncu case)")
    return ap.parse_args()


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=None)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during a timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# CPU baseline (oracle port of the reference path)
# ---------------------------------------------------------------------------

def cpu_layer_sample(n_slots, seed=0, ctx_lo=CTX_LO, ctx_hi=CTX_HI):
    """Builds one decoder layer + N slots on the host and returns a callable
    timing one layer step (all 4 rounds, LoRA, RoPE, attention, norms)."""
    import math
    import torch
    from oracle import reference_math as ref

    torch.manual_seed(seed)
    H, I, HQ, HKV, D, r, s = 4096, 14336, 32, 8, 128, 16, 2.0
    bf = torch.bfloat16
    rnd = lambda *sh: (torch.randn(*sh) * 0.02).to(bf)
    # weights pre-converted to fp32 once (the reference keeps its weights resident)
    Wqkv = ref.fuse_qkv(rnd(HQ * D, H), rnd(HKV * D, H), rnd(HKV * D, H)).float()
    Wo, Wgu, Wd = rnd(H, H).float(), ref.fuse_gate_up(rnd(I, H), rnd(I, H)).float(), rnd(H, I).float()
    w_in = torch.ones(H, dtype=bf)
    ads = []
    for _ in range(n_slots):
        A = {k: rnd(r, i) for k, i in (("q", H), ("k", H), ("v", H), ("o", H), ("g", H), ("u", H), ("d", I))}
        B = {k: rnd(o, r) for k, o in (("q", HQ * D), ("k", HKV * D), ("v", HKV * D), ("o", H), ("g", I), ("u", I), ("d", H))}
        fq = ref.pack_fused_lora([A["q"], A["k"], A["v"]], [B["q"], B["k"], B["v"]], s, [HQ * D, HKV * D, HKV * D])
        fg = ref.pack_fused_lora([A["g"], A["u"]], [B["g"], B["u"]], s, [I, I])
        ads.append((fq, fg, A, B))
    ctx = [int(c) for c in torch.randint(ctx_lo, ctx_hi + 1, (n_slots,))]
    pages_per = (ctx_hi + 16 + 15) // 16
    kc = torch.randn(n_slots * pages_per, 16, HKV, D).to(bf)
    vc = torch.randn(n_slots * pages_per, 16, HKV, D).to(bf)
    tables = [list(range(i * pages_per, (i + 1) * pages_per)) for i in range(n_slots)]
    cs = ref.cos_sin_cache(ref.llama3_inv_freq(D), ctx_hi + 16)
    xs = [torch.randn(1, H).to(bf) for _ in range(n_slots)]

    def mm(xl, W):  # the round: cat -> x @ W^T -> split (ext_aggregator.cpp:545-625)
        rows = [x.shape[0] for x in xl]
        return list(torch.split((torch.cat(xl, 0).float() @ W.t()).to(bf), rows, 0))

    def step(h=None):
        h = xs if h is None else h
        x = [ref.rms_norm(v, w_in) for v in h]
        qkv = mm(x, Wqkv)
        attn = []
        for i in range(n_slots):
            (fA, fB), _, A, B = ads[i]
            parts = [ref.add_bf16(p, d) for p, d in zip(torch.split(qkv[i], [HQ * D, HKV * D, HKV * D], -1),
                                                        ref.fused_lora_delta(x[i], fA, fB, [HQ * D, HKV * D, HKV * D]))]
            pos = torch.tensor([ctx[i]])
            q = ref.rope_neox(parts[0], pos, cs, D)
            k = ref.rope_neox(parts[1], pos, cs, D)
            attn.append(ref.attention_with_kvcache(q.reshape(1, HQ, D), k.reshape(1, HKV, D),
                                                   parts[2].reshape(1, HKV, D), kc, vc, tables[i],
                                                   ctx[i], 1.0 / math.sqrt(D)).reshape(1, HQ * D))
        o = mm(attn, Wo)
        h = [ref.add_bf16(h[i], ref.add_bf16(o[i], ref.lora_delta_scale_after(attn[i], ads[i][2]["o"], ads[i][3]["o"], s)))
             for i in range(n_slots)]
        x = [ref.rms_norm(v, w_in) for v in h]
        gu = mm(x, Wgu)
        act = []
        for i in range(n_slots):
            _, (gA, gB), _, _ = ads[i]
            g, u = torch.split(gu[i], [I, I], -1)
            dg, du = ref.fused_lora_delta(x[i], gA, gB, [I, I])
            act.append(ref.silu_mul(ref.add_bf16(g, dg), ref.add_bf16(u, du)))
        d = mm(act, Wd)
        return [ref.add_bf16(h[i], ref.add_bf16(d[i], ref.lora_delta_scale_after(act[i], ads[i][2]["d"], ads[i][3]["d"], s)))
                for i in range(n_slots)]

    W_lm = []

    def full_step(layers=32):
        """One decode token for every slot: `layers` decoder-layer passes (one
        layer's weights and KV cache reused by every pass: the CPU does the
        same work as with distinct weights), the final norm and the LM-head
        GEMV + argmax (ext_aggregator.cpp:818-861) over a resident fp32
        [128256, 4096] weight."""
        if not W_lm:
            W_lm.append((torch.randn(128256, H) * 0.02).to(bf).float())
        h = xs
        for _ in range(layers):
            h = step(h)
        last = torch.cat([ref.rms_norm(v, w_in) for v in h], 0).float()
        return (last @ W_lm[0].t()).argmax(-1)

    def round_us(m, reps=3):
        """Mean microseconds of one round of each op type (cat -> x @ W^T ->
        split) over m one-row slots."""
        out = {}
        for name, W in (("qkv", Wqkv), ("o", Wo), ("gate_up", Wgu), ("down", Wd)):
            xl = [torch.randn(1, W.shape[1]).to(bf) for _ in range(m)]
            mm(xl, W)
            t0 = time.perf_counter()
            for _ in range(reps):
                mm(xl, W)
            out[name] = round((time.perf_counter() - t0) / reps * 1e6, 1)
        return out

    full_step.round_us = round_us
    return step, full_step


def workload_string(slots, ctx_lo, ctx_hi, layers=32, vocab=128256):
    """The workload both arms name in config.workload."""
    which = 5 if (slots, ctx_lo, ctx_hi) == (32, 1024, 4096) else 2
    return (f"BASELINE config {which}: Llama-3.1-8B shape ({layers} layers, vocab {vocab}), "
            f"{slots} decode slots/GPU, distinct r=16 adapters on 7 projections, "
            f"ctx U[{ctx_lo},{ctx_hi}] paged 16, 1 token/slot/step, greedy")


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_baseline(n_slots, seconds_budget=20.0, ctx_lo=CTX_LO, ctx_hi=CTX_HI):
    """Whole decode steps of the reference's path on the host (oracle/ on
    torch CPU), as many as fit in about `seconds_budget` (at least one)."""
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    _, full_step = cpu_layer_sample(n_slots, ctx_lo=ctx_lo, ctx_hi=ctx_hi)
    full_step(layers=1)  # warm-up (and the LM-head weight)
    times = []
    t_start = time.perf_counter()
    while not times or (time.perf_counter() - t_start + times[-1] < seconds_budget and len(times) < 5):
        t0 = time.perf_counter()
        full_step()
        times.append(time.perf_counter() - t0)
    t_step = sum(times) / len(times)
    # the per-round metric on the same cores: M = the slots (one row each) and
    # M = 4 (the reference's CPU-runnable one-layer configuration)
    rounds = {"m%d" % m: full_step.round_us(m) for m in (n_slots, 4)}
    return {"value": round(n_slots / t_step, 4), "unit": UNIT, "cores": threads, "cpu": cpu_model(),
            "us_per_round": rounds,
            "kind": "port",
            "sample": f"{len(times)} whole decode steps of {n_slots} slots at ctx U[{ctx_lo},{ctx_hi}] "
                      f"(32 layer passes: 4 rounds + LoRA + RoPE + paged attention + norms; one layer's "
                      f"weights reused; LM-head GEMV + argmax), mean {t_step * 1e3:.0f} ms; oracle/ on torch "
                      f"CPU, {threads} threads"}


def reference_arm(args):
    """The reference's path on the host cores (the oracle restatement on
    torch CPU, every thread): each step is one whole decode token for every
    slot (32 layer passes + LM head), so ms_per_step is the timed step."""
    import torch
    world, rank, _ = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    _, full_step = cpu_layer_sample(args.slots, ctx_lo=args.ctx_lo, ctx_hi=args.ctx_hi)
    full_step(layers=1)
    for _ in range(args.warmup):
        full_step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        full_step()
        times.append(time.perf_counter() - t0)
    t_step = sum(times) / len(times)
    value = args.slots / t_step
    rounds = {"m%d" % m: full_step.round_us(m) for m in (args.slots, 4)}
    sample = (f"{args.steps} whole decode steps of {args.slots} slots (32 layer passes with one layer's weights "
              f"reused + LM-head GEMV + argmax) on {threads} threads")
    line = {"metric": metric_for(args.slots), "value": round(value, 4), "unit": UNIT, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_step * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload_string(args.slots, args.ctx_lo, args.ctx_hi),
                       "slots": args.slots, "layers": 32, "vocab": 128256, "sample": sample},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "cpu": cpu_model(),
                             "kind": "port", "sample": sample, "us_per_round": rounds},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def round_phase(grp, cfg, reps=3, rows=None):
    """Times each round kind over all layers' weights (> L2 in total) from a
    CUDA graph; returns {op: us per launch} and the algorithmic bytes. `rows`
    gives each slot's token rows (default one)."""
    import torch
    from swarmlora_b200 import ext_aggregator as agg
    from swarmlora_b200._native import i64_array
    ops = {"qkv": agg.OP_QKV_FUSED, "o": agg.OP_O_PROJ, "gate_up": agg.OP_GATE_UP_FUSED,
           "down": agg.OP_DOWN_PROJ}
    tx = i64_array(rows) if rows is not None else None
    H, I, M = cfg.hidden, cfg.inter, (sum(rows) if rows is not None else grp.n)
    shapes = {"qkv": (cfg.qkv_n, H), "o": (H, cfg.hq * cfg.head_dim), "gate_up": (2 * I, H), "down": (H, I)}
    s = torch.cuda.Stream()
    out = {}
    for name, op in ops.items():
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for l in range(cfg.layers):
                grp._round(op, l, s.cuda_stream, tx)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        with torch.cuda.stream(s):
            for _ in range(reps):
                g.replay()
        b.record(s)
        b.synchronize()
        us = a.elapsed_time(b) * 1e3 / (reps * cfg.layers)
        N, K = shapes[name]
        byts = 2 * N * K + 2 * M * K + 2 * M * N
        out[name] = {"us": round(us, 3), "bytes": byts, "gbs": round(byts / us / 1e3, 1)}
        del g
    return out


def protocol_phase(grp, args, variants, rounds=None):
    """Decode through the drop-in protocol: the aggregator's main loop
    serving native worker clients (swarmlora_b200.protocol) that request
    every round through the shared-memory ring and epoch barrier, as the
    reference's workers do. `variants`: (workers, completion, input_ready, per-segment graphs).
    Returns one dict per variant: tok/s over the timed tokens (host clock of
    the slowest client, from each token's first launch to its last round's
    epoch), and per-round times."""
    import statistics
    import torch
    from swarmlora_b200.protocol import ProtocolRun
    n = grp.n
    ops = 1 + 4 * grp.cfg.layers + 1
    out = []
    for workers, completion, input_ready, graphs in variants:
        grp.reset_positions()
        torch.cuda.synchronize()
        run = ProtocolRun(grp, workers=workers, completion=completion, input_ready=input_ready, graphs=graphs)
        try:
            res = run.run(args.warmup + args.steps)
        finally:
            run.close()
        timed = res["token_s"][args.warmup:]
        tok_s = n * len(timed) / sum(timed)
        entry = {"workers": workers, "slots_per_worker": round(n / workers, 2), "completion": completion,
                 "input_ready": input_ready, "segment_graphs": graphs, "tok_s": round(tok_s, 2),
                 "ms_per_token": round(1e3 * sum(timed) / len(timed), 3),
                 "ms_per_token_p50": round(1e3 * statistics.median(timed), 3),
                 "us_per_round_e2e": round(1e6 * sum(timed) / len(timed) / ops, 2)}
        if rounds:
            entry["us_per_round_kernels"] = round(
                (sum(v["us"] for v in rounds.values()) * grp.cfg.layers) / (4 * grp.cfg.layers), 2)
        out.append(entry)
    grp.reset_positions()
    return out


def our_arm(args):
    import torch
    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import dataclasses
    from swarmlora_b200.engine import LLAMA_3_1_8B, SlotGroup, random_adapter, random_base

    import swarmlora_b200
    swarmlora_b200.set_pdl(not args.no_pdl)
    from swarmlora_b200 import worker_ops as _wo
    _wo.attention_tune(args.attn_chunk_pages, args.attn_stages, args.attn_groups)
    _wo.attention_tma(not args.attn_lane_copies)
    if args.round_flags or args.round_tile:
        from swarmlora_b200._native import check as _check, lib as _lib
        bn, st = (int(x) for x in args.round_tile.split("x")) if args.round_tile else (0, 0)
        _check(_lib().swl_round_tune(32, bn, st, args.round_flags))
    if args.checkpoint:
        from swarmlora_b200.checkpoint import load_base
        base, cfg = load_base(args.checkpoint, dev)
    else:
        cfg = dataclasses.replace(LLAMA_3_1_8B, layers=args.layers, vocab=args.vocab)
        base = random_base(cfg, seed=1, device=dev)
    n = args.slots
    g = torch.Generator().manual_seed(1234 + rank)
    ctx = [int(c) for c in torch.randint(args.ctx_lo, args.ctx_hi + 1, (n,), generator=g)]
    adapters = [random_adapter(cfg, seed=100 + rank * 1000 + i, device=dev) for i in range(n)]
    total_new = args.warmup + args.steps + args.warmup + args.steps + 4
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=max(MAX_NEW, total_new), device=local, seed=rank)
    start_tokens = torch.randint(0, cfg.vocab, (n,), generator=g)
    grp.tokens.copy_(start_tokens)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        grp.enqueue_step(stream)  # eager warm-up (sets kernel attributes before capture)
    torch.cuda.synchronize()
    grp.reset_positions()
    grp.tokens.copy_(start_tokens)
    grp.capture(stream)

    # ---- device-resident throughput -------------------------------------------
    for _ in range(args.warmup):
        grp.replay()
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.25)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            if args.profile_step and i == 0:
                torch.cuda.profiler.start()
            grp.replay()
            if args.profile_step and i == 0:
                torch.cuda.synchronize()
                torch.cuda.profiler.stop()
    ev1.record(stream)
    ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    time.sleep(0.1)
    clk = clocks.stop()
    torch.cuda.synchronize()
    barrier(world)
    ms_max = max_over_ranks(ms, world, dev)
    value = n * world * args.steps / (ms_max / 1e3)

    # ---- end to end: host token ids in, next tokens out, every step --------------
    grp.reset_positions()
    h_in = torch.empty(n, dtype=torch.int64).pin_memory()
    h_out = torch.empty(n, dtype=torch.int64).pin_memory()
    h_in.copy_(grp.tokens.cpu())
    for _ in range(args.warmup):
        grp.tokens.copy_(h_in, non_blocking=True)
        grp.replay()
        h_out.copy_(grp.tokens, non_blocking=True)
        torch.cuda.synchronize()
        h_in.copy_(h_out)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            grp.tokens.copy_(h_in, non_blocking=True)
            grp.replay()
            h_out.copy_(grp.tokens, non_blocking=True)
            stream.synchronize()
            h_in.copy_(h_out)
    e1.record(stream)
    e1.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    e2e = n * world * args.steps / (e2e_ms / 1e3)

    # ---- per-round kernel times (roofline of the dominant kernel) --------------
    # DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one round
    # launch at this workload, from the capture
    #   ncu --set full --clock-control none -k regex:slot_round -s 1 -c 1 \
    #       python bench.py --profile-round gate_up --steps 3 --warmup 1
    ncu_traffic = {("gate_up", 28): 235_173_376 + 4_176_640}
    rounds = round_phase(grp, cfg)
    proto = None
    if args.protocol != "off" and world == 1:
        variants = []
        for w in (int(x) for x in args.protocol.split(",")):
            w = min(max(1, w), n)
            variants += [(w, "event", "event", True), (w, "event", "event", False), (w, "host", "sync", False)]
        proto = protocol_phase(grp, args, variants, rounds)
    peak, peak_kind = measured_peaks()
    dom = max(rounds, key=lambda k: rounds[k]["us"])
    achieved = rounds[dom]["bytes"] / rounds[dom]["us"] / 1e3
    launches = grp.launches_per_step() * args.steps

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline(n, ctx_lo=args.ctx_lo, ctx_hi=args.ctx_hi)
        except Exception as e:  # report, do not fail the GPU number
            cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {e}"}

    if rank == 0:
        line = {
            "metric": metric_for(args.slots), "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": ("base weights from " + os.path.basename(os.path.normpath(args.checkpoint))
                     + "; synthetic adapters and KV contexts") if args.checkpoint
                    else "synthetic (seeded random-init weights, adapters, KV contexts)",
            "config": {"workload": workload_string(n, args.ctx_lo, args.ctx_hi, cfg.layers, cfg.vocab),
                       "slots_per_gpu": n, "parallelism": f"{world} independent aggregator groups",
                       "launch": "serialized" if args.no_pdl else "programmatic dependent launch",
                       "l2": "weights (15 GB/step) far exceed L2; no flush needed",
                       "us_per_round": {k: v["us"] for k, v in rounds.items()},
                       "round_gbs": {k: v["gbs"] for k, v in rounds.items()}},
            "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": 8 * n,
                    "d2h_bytes_per_step": 8 * n},
            "roofline": {"bound": "hbm", "kernel": f"slot_round_tc ({dom} round, M={n})",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": ncu_traffic.get((dom, n)),
                         "traffic_unit": "bytes/launch", "algorithmic_bytes": rounds[dom]["bytes"],
                         "peak_source": peak_kind},
            "gpu_launches": launches,
            "clocks": clk,
        }
        if proto:
            # the same decode through the drop-in protocol: the reference's
            # deployment shape (main loop + worker clients over the shm ring)
            line["e2e_protocol"] = proto
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    grp.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def profile_round(args):
    """Standalone round case for kernel captures: one weight of the named round
    (> L2 for gate_up/down), --slots decode slots, --steps launches."""
    import torch
    from swarmlora_b200.rounds import slot_gemm
    H, I = 4096, 14336
    N, K = {"qkv": (6144, H), "o": (H, H), "gate_up": (2 * I, H), "down": (H, I)}[args.profile_round]
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    W = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    rows = max(1, args.round_rows)
    ins = [torch.randn(max(16, rows), K, generator=g, device=dev).to(torch.bfloat16)[:rows] for _ in range(args.slots)]
    outs = [torch.empty(max(16, rows), N, dtype=torch.bfloat16, device=dev) for _ in range(args.slots)]
    for _ in range(args.warmup):
        slot_gemm(W, ins, outs, algo=args.round_algo)
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        slot_gemm(W, ins, outs, algo=args.round_algo)
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    M = args.slots * rows
    us = min(times)
    print(json.dumps({"profile_round": args.profile_round, "M": M, "N": N, "K": K, "launches": args.steps,
                      "us_per_launch_best": round(us, 2), "us_per_launch_all": [round(t, 1) for t in times],
                      "tflops_best": round(2 * M * N * K / us / 1e6, 1)}))
    return 0


def profile_attention(args):
    """Standalone decode attention case: --slots rows, contexts U[256,1024],
    one layer of paged KV; --steps launches of attention + combine captured in
    a CUDA graph, cycling over 4 cache copies (4 x ~120 MB > L2)."""
    import math
    import torch
    from swarmlora_b200 import worker_ops as wo
    from swarmlora_b200.engine import LLAMA_3_1_8B as cfg
    wo.attention_tune(args.attn_chunk_pages, args.attn_stages, args.attn_groups)
    wo.attention_tma(not args.attn_lane_copies)
    dev = torch.device("cuda:0")
    n = args.slots
    g = torch.Generator(device=dev).manual_seed(0)
    ctx = [int(c) for c in torch.randint(CTX_LO, CTX_HI + 1, (n,), generator=torch.Generator().manual_seed(1))]
    pps = (CTX_HI + 1 + 15) // 16
    perm = torch.randperm(n * pps, generator=g, device=dev).to(torch.int32)
    bts = [perm[i * pps:(i + 1) * pps].contiguous() for i in range(n)]
    caches = [(torch.randn(n * pps, 16, cfg.hkv, cfg.head_dim, generator=g, device=dev).to(torch.bfloat16),
               torch.randn(n * pps, 16, cfg.hkv, cfg.head_dim, generator=g, device=dev).to(torch.bfloat16))
              for _ in range(4)]
    sl = torch.tensor(ctx, dtype=torch.int32, device=dev)
    q = torch.randn(n, cfg.hq * cfg.head_dim, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    part = torch.empty(wo.attention_part_floats(n, cfg.hq, cfg.hkv, CTX_HI + 1), dtype=torch.float32, device=dev)

    def call(i):
        kc, vc = caches[i % len(caches)]
        wo.paged_attention([1] * n, bts, [kc] * n, [vc] * n, [sl[j:j + 1] for j in range(n)],
                           [out[j:j + 1] for j in range(n)], q, part, cfg.hq, cfg.hkv, CTX_HI + 1,
                           1.0 / math.sqrt(cfg.head_dim))
    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize()
    st = torch.cuda.Stream(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for i in range(args.steps):
            call(i)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for _ in range(3):
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        best = min(best, a.elapsed_time(b) * 1e3 / args.steps)
    kv_bytes = sum(ctx) * cfg.hkv * cfg.head_dim * 2 * 2
    print(json.dumps({"profile_attention": True, "rows": n, "kv_bytes": kv_bytes, "us_per_call": round(best, 2),
                      "gbs": round(kv_bytes / best / 1e3, 1), "chunk_pages": args.attn_chunk_pages,
                      "stages": args.attn_stages}))
    return 0


def shard_arm(args):
    """The multi-GPU configuration's column-sharded variant: ONE slot group
    served by two GPUs, each holding half of every fused weight's output
    columns and writing them into both GPUs' slot outputs from the round
    epilogue (peer stores over NVLink). Prints one JSON line (rank 0)."""
    import torch
    world, rank, local = dist_setup(args.gpus)
    if world != 2:
        print(json.dumps({"shard": "unavailable", "why": "needs torchrun with 2 ranks (--gpus 2)"}))
        return 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import dataclasses
    from swarmlora_b200.engine import LLAMA_3_1_8B, SlotGroup, random_adapter, random_base
    cfg = dataclasses.replace(LLAMA_3_1_8B, layers=args.layers, vocab=args.vocab)
    n = args.slots
    g = torch.Generator().manual_seed(1234)  # the same group on both GPUs
    ctx = [int(c) for c in torch.randint(CTX_LO, CTX_HI + 1, (n,), generator=g)]
    base = random_base(cfg, seed=1, device=dev)
    adapters = [random_adapter(cfg, seed=100 + i, device=dev) for i in range(n)]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=MAX_NEW + args.warmup + args.steps, device=local, seed=0)
    grp.shard(rank)
    start_tokens = torch.randint(0, cfg.vocab, (n,), generator=g)
    grp.tokens.copy_(start_tokens)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        grp.enqueue_step(stream)
    torch.cuda.synchronize()
    grp.reset_positions()
    grp.tokens.copy_(start_tokens)
    grp.capture(stream)
    for _ in range(args.warmup):
        grp.replay()
    torch.cuda.synchronize()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            grp.replay()
    ev1.record(stream)
    ev1.synchronize()
    ms_max = max_over_ranks(ev0.elapsed_time(ev1), world, dev)
    rounds = round_phase(grp, cfg)
    from swarmlora_b200 import rounds as R
    err = R.device_error()
    toks = grp.tokens.cpu()
    both = [None, None]
    import torch.distributed as dist
    dist.all_gather_object(both, toks.tolist())
    if rank == 0:
        print(json.dumps({
            "metric": metric_for(args.slots) + " (column-sharded base weights, one group on 2 GPUs)",
            "value": round(n * args.steps / (ms_max / 1e3), 2), "unit": UNIT, "n_gpus": 2,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic (seeded random-init weights, adapters, KV contexts)",
            "config": {"workload": f"Llama-3.1-8B shape ({cfg.layers} layers, vocab {cfg.vocab}), {n} decode slots "
                                   f"in one group, ctx U[{CTX_LO},{CTX_HI}]",
                       "parallelism": "column-sharded base weights x2, outputs all-gathered by peer stores "
                                      "from the round epilogue",
                       "us_per_round": {k: v["us"] for k, v in rounds.items()}},
            "ranks_agree": both[0] == both[1], "device_error": err}), flush=True)
    grp.close()
    dist.destroy_process_group()
    return 0


def mixed_arm(args):
    """BASELINE config 3 on one GPU: 28 slots of the 8B shape, 4 of them
    prefilling prompts of U[512, 2048] tokens in chunks of --mixed-chunk rows
    per step (a prompt that is done starts over as a new request) beside 24
    decode slots at contexts U[256, 2048]; every step's rounds carry
    4 * chunk + 24 rows. The step is a CUDA graph of the fixed row pattern;
    each step first stages the prefill chunks' token ids into the group's
    token buffer. value = new tokens (prefill + decode) per second; e2e adds
    the chunks' ids from pinned host memory and reads the next tokens back
    every step. Each prefill slot starts at a seeded chunk boundary inside
    its prompt (its prefix already in the cache), so the prefixes attended to
    spread over the prompt lengths. Prints one JSON line."""
    import dataclasses
    import torch
    import swarmlora_b200
    from swarmlora_b200.engine import LLAMA_3_1_8B, SlotGroup, random_adapter, random_base
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    swarmlora_b200.set_pdl(not args.no_pdl)
    chunk, n_pf, n_dec = int(args.mixed_chunk), 4, 24
    n = n_pf + n_dec
    if not 1 <= chunk or n_pf * chunk + n_dec > 256:
        raise SystemExit("--mixed-chunk: 4 * chunk + 24 rows must stay within 256")
    cfg = dataclasses.replace(LLAMA_3_1_8B, layers=args.layers, vocab=args.vocab, max_seq_per_step=chunk)
    g = torch.Generator().manual_seed(4321)
    prompts = [(int(x) + chunk - 1) // chunk * chunk for x in torch.randint(512, 2049, (n_pf,), generator=g)]
    dec_ctx = [int(c) for c in torch.randint(256, 2049, (n_dec,), generator=g)]
    steps_total = args.warmup + args.steps
    base = random_base(cfg, seed=1, device=dev)
    adapters = [random_adapter(cfg, seed=300 + i, device=dev) for i in range(n)]
    # each prefill slot starts at a seeded chunk boundary inside its prompt, so
    # the prefixes its rows attend to cover the prompt lengths as a steady
    # stream of prefilling requests does (not only their first chunks)
    offs = [chunk * int(torch.randint(0, (p_len - chunk) // chunk + 1, (1,), generator=g)) for p_len in prompts]
    grp = SlotGroup(cfg, base, adapters, offs + dec_ctx,
                    max_new=max(max(prompts), 2 * steps_total + 8), device=0, seed=0)
    rows = [chunk] * n_pf + [1] * n_dec
    ids = torch.randint(0, cfg.vocab, (n_pf, max(prompts)), generator=g)
    ids_dev = ids.to(dev)
    grp.tokens.copy_(torch.randint(0, cfg.vocab, (n,), generator=g))
    stream = torch.cuda.Stream(dev)
    done = list(offs)  # prefilled tokens of each prefill slot's current prompt

    def stage(host_ids=None):
        """Token ids of the next step into tok_in (decode rows: last outputs)."""
        grp.tok_in[:, 0].copy_(grp.tokens)
        for i in range(n_pf):
            if done[i] + chunk > prompts[i]:  # prompt done: a new request on this slot
                done[i] = 0
                grp.set_context(i, 0)
            src = host_ids[i] if host_ids is not None else ids_dev[i, done[i]:done[i] + chunk]
            grp.tok_in[i, :chunk].copy_(src, non_blocking=True)
            done[i] += chunk
    with torch.cuda.stream(stream):
        stage()
        grp.enqueue_step(stream, rows=rows, tokens=[grp.tok_in[i, :x].tolist() for i, x in enumerate(rows)])
    torch.cuda.synchronize()
    grp.capture(stream, rows=rows)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            stage()
            grp.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    clocks.start()
    time.sleep(0.25)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            stage()
            grp.replay()
    ev1.record(stream)
    ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    time.sleep(0.1)
    clk = clocks.stop()
    new_rows = sum(rows)
    value = new_rows * args.steps / (ms / 1e3)

    # end to end: the chunks' ids from pinned host memory, next tokens back
    h_ids = torch.empty(n_pf, chunk, dtype=torch.int64).pin_memory()
    h_out = torch.empty(n, dtype=torch.int64).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            for i in range(n_pf):
                d = done[i] if done[i] + chunk <= prompts[i] else 0
                h_ids[i].copy_(ids[i, d:d + chunk])
            stage(host_ids=h_ids)
            grp.replay()
            h_out.copy_(grp.tokens, non_blocking=True)
            stream.synchronize()
    e1.record(stream)
    e1.synchronize()
    e2e = new_rows * args.steps / (e0.elapsed_time(e1) / 1e3)

    rounds = round_phase(grp, cfg, rows=rows)
    peak, peak_kind = measured_peaks()
    dom = max(rounds, key=lambda k: rounds[k]["us"])
    achieved = rounds[dom]["bytes"] / rounds[dom]["us"] / 1e3
    line = {
        "metric": "mixed prefill+decode new tokens/s/GPU (Llama-3.1-8B shape, 4 prefill + 24 decode slots)",
        "value": round(value, 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights, adapters, prompts)",
        "config": {"workload": f"BASELINE config 3: {cfg.layers} layers, vocab {cfg.vocab}; 4 slots prefilling "
                               f"prompts U[512,2048] in {chunk}-row chunks (each from a seeded point inside its "
                               f"prompt) + 24 decode slots at ctx U[256,2048], "
                               f"{new_rows} rows per round, distinct r=16 adapters",
                   "prefill_tok_s": round(n_pf * chunk * args.steps / (ms / 1e3), 2),
                   "decode_tok_s": round(n_dec * args.steps / (ms / 1e3), 2),
                   "l2": "weights (15 GB/step) far exceed L2; no flush needed",
                   "us_per_round": {k: v["us"] for k, v in rounds.items()},
                   "round_gbs": {k: v["gbs"] for k, v in rounds.items()}},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 8 * n_pf * chunk,
                "d2h_bytes_per_step": 8 * n},
        "roofline": {"bound": "hbm", "kernel": f"slot_round_tc ({dom} round, M={new_rows})",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "algorithmic_bytes": rounds[dom]["bytes"], "peak_source": peak_kind},
        # the mixed step advances its positions with a torch add, not this
        # library's advance kernel
        "gpu_launches": (grp.launches_per_step() - 1) * args.steps,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    grp.close()
    return 0


def profile_layers_arm(args):
    """The decode workload (--slots, --ctx-lo/--ctx-hi, --layers, --vocab)
    stepped eagerly with a CUDA event after every launch; prints one
    [LAYER_PROFILE] line per step (SlotGroup.profile_step)."""
    import dataclasses
    import torch
    from swarmlora_b200.engine import LLAMA_3_1_8B, SlotGroup, random_adapter, random_base
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = dataclasses.replace(LLAMA_3_1_8B, layers=args.layers, vocab=args.vocab)
    n = args.slots
    g = torch.Generator().manual_seed(1234)
    ctx = [int(c) for c in torch.randint(args.ctx_lo, args.ctx_hi + 1, (n,), generator=g)]
    base = random_base(cfg, seed=1, device=dev)
    adapters = [random_adapter(cfg, seed=100 + i, device=dev) for i in range(n)]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=args.profile_layers + 8, device=0, seed=0)
    grp.tokens.copy_(torch.randint(0, cfg.vocab, (n,), generator=g))
    grp.profile_step(print_line=False)  # kernel attributes, first-launch costs
    for _ in range(args.profile_layers):
        grp.profile_step(print_line=True)
    grp.close()
    return 0


def churn_arm(args):
    """The churn configuration on one GPU: a seeded trace of Poisson arrivals
    (8/s), lognormal prompts and outputs, Zipf adapter ids over a pool of 500
    adapters of ranks 8/16/32 (random-init, made on the device when missed,
    or with --churn-from-disk read from PEFT adapter files written before the
    run), an LRU cache of 32 of them packed into slabs (a swap is one device
    copy), prefill in 16-row chunks next to decode rows
    (at most 256 rows a step), all-decode steps replayed from a CUDA graph.
    The clock is the device time of steps and swaps. Prints one JSON line."""
    import dataclasses
    import torch
    from swarmlora_b200.churn import ChurnConfig, ChurnRunner, adapter_ranks, make_trace
    from swarmlora_b200.engine import LLAMA_3_1_8B, SlotGroup, random_adapter, random_base
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ccfg = ChurnConfig()
    cfg = dataclasses.replace(LLAMA_3_1_8B, layers=args.layers, vocab=args.vocab, rank=max(ccfg.ranks))
    ranks = adapter_ranks(ccfg)

    n = args.churn_slots
    base = random_base(cfg, seed=1, device=dev)
    a0 = random_adapter(cfg, seed=10_000, device=dev, rank=int(ranks[0]))
    grp = SlotGroup(cfg, base, [a0] * n, [0] * n, max_new=ccfg.prompt_clip[1] + ccfg.output_clip[1] + 16,
                    device=0, seed=0)

    trace = make_trace(ccfg, args.churn, seed=0)
    loader, pool_dir = None, None
    if args.churn_from_disk:  # every adapter the trace uses, as a bf16 PEFT directory
        import shutil
        from swarmlora_b200.adapters import AdapterLoader, save_adapter
        pool_dir = str(ROOT / "_build" / f"adapter_pool_{os.getpid()}")  # inside the checkout (ignored by git)
        shutil.rmtree(pool_dir, ignore_errors=True)
        os.makedirs(pool_dir)
        for aid in sorted({r.adapter for r in trace}):
            save_adapter(os.path.join(pool_dir, f"lora-{aid}"),
                         random_adapter(cfg, seed=10_000 + aid, device=dev, rank=int(ranks[aid])),
                         alpha=cfg.alpha, dtype=torch.bfloat16)
        loader = AdapterLoader(cfg, dev, allowed_bases=[pool_dir])

    def load(aid):
        """A miss: read the adapter's files (pinned staging, one copy to the
        GPU) or make it on the device, then pack it into a slab."""
        if loader is not None:
            layers, conf = loader.load(os.path.join(pool_dir, f"lora-{aid}"))
            return grp.pack_adapter(layers, scaling=conf["scaling"])
        return grp.pack_adapter(random_adapter(cfg, seed=10_000 + aid, device=dev, rank=int(ranks[aid])))
    stream = torch.cuda.Stream(dev)

    def timer(fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / 1e3
    with torch.cuda.stream(stream):
        grp.enqueue_step(stream)  # kernel attributes before capture
    torch.cuda.synchronize()
    for i in range(n):
        grp.set_context(i, 0)
    grp.capture(stream)
    st = ChurnRunner(grp, trace, ccfg, load, timer, cfg.vocab, stream=stream).run()
    if pool_dir:
        shutil.rmtree(pool_dir, ignore_errors=True)
    print(json.dumps({"metric": "churn: decode tokens per device second (Llama-3.1-8B shape)",
                      "requests": len(trace), **st.summary(), "dtype": "bf16",
                      "config": {"workload": f"{args.churn:g} s of arrivals at {ccfg.rate}/s, pool {ccfg.pool_size} "
                                             f"adapters r in {list(ccfg.ranks)}, cache {ccfg.cache_adapters}, "
                                             f"{n} slots, {cfg.layers} layers, vocab {cfg.vocab}, "
                                             f"misses {'read from PEFT files' if loader else 'made on the device'}",
                                 "data": "synthetic (seeded trace, random-init weights and adapters)"}}), flush=True)
    grp.close()
    return 0


def main():
    args = parse()
    if args.profile_layers:
        return profile_layers_arm(args)
    if args.churn:
        return churn_arm(args)
    if args.mixed:
        return mixed_arm(args)
    if args.shard:
        return shard_arm(args)
    if args.profile_attention:
        return profile_attention(args)
    if args.profile_round:
        return profile_round(args)
    if args.impl == "reference":
        return reference_arm(args)
    return our_arm(args)


if __name__ == "__main__":
    sys.exit(main())
