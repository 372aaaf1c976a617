"""The reference's deployment shape on one GPU: the aggregator's main loop
(ext_aggregator.aggregator_main_loop_slots, ext_aggregator.cpp:1024-1210)
serving adapter workers that request every round through the shared-memory
command ring and epoch barrier (worker_sync.py:230-389, 1274-1425).

`ProtocolRun` takes a `SlotGroup` (which owns the slot pool, the fused base
weights and every slot's adapter, KV cache and hidden rows) and splits its
slots over W native worker clients (`swl_wc_*`, one host thread each). Each
client runs the reference worker's per-token loop for its slots with this
library's worker kernels, and the aggregator thread runs the main loop; the
rounds are the same kernels the in-process engine launches, now requested
through the protocol. With W equal to the slot count every worker owns one
slot, as in the reference (MAX_CONCURRENT_REQUESTS_PER_WORKER=1,
config.py:46); fewer workers own several slots each (the reference's worker
API takes up to 8 slots per worker, ext_unified_barrier.cpp:22).

Completion of a round on the aggregator side: "host" synchronizes the
stream and bumps the epoch (the reference); "device" has the GPU store the
epoch after the round (swl_agg_set_completion_mode(1)). A client learns that
its round input is written either by a stream sync ("sync", as
prepare_input_slot) or from a device-written host flag ("flag"). "event"
(with input_ready "event") orders both directions by CUDA events instead:
a client records an event after writing its inputs and sets its ready bits
at once, the aggregator's stream waits for those events, and the epoch
moves as soon as the round is enqueued; the client's stream then waits for
the round's event. No host thread waits for the GPU inside a token. With
`graphs` (event completion only) each client captures the launches between
two rounds, event wait and record included, into one CUDA graph after its
first token, and the aggregator replays each round (its input-event waits,
kernels and round-event record) from a graph once the same command set
repeats, so a round costs each client and the aggregator one launch.
"""
from __future__ import annotations

import ctypes as C
import threading
import time

import torch

from . import ext_aggregator as agg
from . import ext_ipc_queue as extq
from . import worker_ops as wo
from ._native import check, i32_array, lib, ptr_array


class ProtocolRun:
    def __init__(self, grp, workers: int, completion: str = "device", input_ready: str = "flag",
                 timeout_ms: int = 30000, capacity: int = 512, graphs: bool = False):
        if (completion, input_ready) not in (("host", "sync"), ("host", "flag"), ("device", "sync"),
                                             ("device", "flag"), ("event", "event")):
            raise ValueError("completion 'host' or 'device' with input_ready 'sync' or 'flag', "
                             "or completion 'event' with input_ready 'event'")
        if not grp.fused or grp._subset is not None:
            raise ValueError("the protocol clients run a full group's fused sequence")
        n = grp.n
        if not 1 <= workers <= n:
            raise ValueError(f"workers must be 1..{n}")
        self.grp, self.workers = grp, workers
        self.completion, self.input_ready = completion, input_ready
        cfg = grp.cfg
        L = lib()
        # the queue: this process is both the workers' side (swl_q_*) and the aggregator's
        info = extq.create_queue(capacity, capacity)
        self._queue_open = True
        agg.init_aggregator_queue(info["shm_name"], capacity)
        extq.init_batch_control(n)
        check(L.swl_agg_set_completion_mode({"host": 0, "device": 1, "event": 2}[completion]))
        # with graphs, the aggregator also replays each round from a graph
        check(L.swl_agg_set_round_graphs(1 if graphs else 0))
        # contiguous slot ranges, as even as possible
        bounds = [round(i * n / workers) for i in range(workers + 1)]
        self.ranges = [(bounds[i], bounds[i + 1]) for i in range(workers)]
        self._keep = []  # ctypes arrays and scratch tensors the clients point into
        self.handles = []
        dev = grp.dev
        D, r = cfg.head_dim, cfg.rank
        for a, b in self.ranges:
            k = b - a
            idx = list(range(a, b))
            h = C.c_void_p()
            check(L.swl_wc_create(k, i32_array([grp.slot_ids[i] for i in idx]),
                                  i32_array([grp.worker_ids[i] for i in idx]), cfg.layers, cfg.hidden, cfg.inter,
                                  cfg.hq, cfg.hkv, D, cfg.page, r, cfg.eps, grp.scaling, grp.max_len, C.byref(h)))
            self.handles.append(h)
            f32 = dict(dtype=torch.float32, device=dev)
            scratch = dict(
                q_rot=torch.empty(k * grp.max_rows, cfg.hq * D, dtype=torch.bfloat16, device=dev),
                part=torch.empty(max(1, wo.attention_part_floats(k * grp.max_rows, cfg.hq, cfg.hkv, grp.max_len)),
                                 **f32),
                ws_qkv=torch.zeros(grp.norm_splits * k * grp.max_rows * 3 * r, **f32),
                ws_o=torch.zeros(cfg.hq * k * grp.max_rows * r, **f32),
                ws_gu=torch.zeros(grp.norm_splits * k * grp.max_rows * 2 * r, **f32),
                ws_dn=torch.zeros(grp.dn_splits * k * grp.max_rows * r, **f32))

            def sub(ptrs):
                return ptr_array([ptrs[i] for i in idx])
            arrs = dict(slot_in=sub(grp.a_in), slot_out=sub(grp.a_out), h=sub(grp.a_h), tok=sub(grp.a_tok),
                        bt=sub(grp.a_bt), sl=sub(grp.a_sl))
            self._keep += [scratch, arrs]
            check(L.swl_wc_set_buffers(h, arrs["slot_in"], arrs["slot_out"], arrs["h"], arrs["tok"], arrs["bt"],
                                       arrs["sl"], grp.seqlens[a].data_ptr(), scratch["q_rot"].data_ptr(),
                                       scratch["part"].data_ptr(), scratch["ws_qkv"].data_ptr(),
                                       scratch["ws_o"].data_ptr(), scratch["ws_gu"].data_ptr(),
                                       scratch["ws_dn"].data_ptr(), grp.cos_sin.data_ptr(),
                                       grp.base.final_norm.data_ptr()))
            for l in range(cfg.layers):
                lay = dict(kc=ptr_array([grp.k_cache[l].data_ptr()] * k), vc=ptr_array([grp.v_cache[l].data_ptr()] * k))
                for name in ("A_qkv", "B_qkv", "A_o", "B_o", "A_gu", "B_gu", "A_dn", "B_dn"):
                    lay[name] = sub(getattr(grp, name)[l])
                self._keep.append(lay)
                check(L.swl_wc_set_layer(h, l, grp.base.in_norm[l].data_ptr(), grp.base.post_norm[l].data_ptr(),
                                         lay["kc"], lay["vc"], lay["A_qkv"], lay["B_qkv"], lay["A_o"], lay["B_o"],
                                         lay["A_gu"], lay["B_gu"], lay["A_dn"], lay["B_dn"]))
            check(L.swl_wc_configure(h, self._input_mode(input_ready), timeout_ms, None))
            if graphs:
                if completion != "event":
                    raise ValueError("per-segment graphs need event completion")
                check(L.swl_wc_use_graphs(h, 1))
        self.graphs = bool(graphs)
        self.timeout_ms = timeout_ms
        self._loop = None
        self._loop_err = []

    @staticmethod
    def _input_mode(input_ready: str) -> int:
        return {"sync": 0, "flag": 1, "event": 2}[input_ready]

    def _start_loop(self):
        grp = self.grp
        for s in grp.slot_ids:
            extq.slot_signal_join(s)

        def run():
            try:
                agg.aggregator_main_loop_slots(grp.n, 15)
            except Exception as e:  # reported by run()
                self._loop_err.append(e)
        self._loop = threading.Thread(target=run, daemon=True)
        self._loop.start()
        t0 = time.time()
        while not all(extq.slot_is_active(s) for s in grp.slot_ids):
            if self._loop_err or time.time() - t0 > self.timeout_ms / 1e3:
                raise RuntimeError(f"slots did not become active: {self._loop_err}")
            time.sleep(0.001)

    def run(self, tokens: int, record: bool = False) -> dict:
        """Every client decodes `tokens` tokens for its slots (in lock-step
        through the aggregator's barrier); returns per-token host times
        (the slowest client's, seconds) and, with `record`, each token's
        picks [tokens, n] (int64, device)."""
        grp, L = self.grp, lib()
        torch.cuda.synchronize(grp.dev)
        if self._loop is None:
            self._start_loop()
        # each client writes its picks as [tokens, its slot count]
        hist_c = [torch.zeros(tokens, b - a, dtype=torch.int64, device=grp.dev) for a, b in self.ranges] \
            if record else None
        bufs, errs = [], []
        for i, h in enumerate(self.handles):
            hp = C.c_void_p(hist_c[i].data_ptr()) if record else None
            check(L.swl_wc_configure(h, self._input_mode(self.input_ready), self.timeout_ms, hp))
            bufs.append((C.c_int64 * max(1, tokens))())

        def client(i):
            st = L.swl_wc_run(self.handles[i], tokens, bufs[i])
            if st != 0:
                from ._native import last_error
                errs.append(f"client {i}: {last_error()}")
                extq.set_quit(1)  # release the others and the loop
        ths = [threading.Thread(target=client, args=(i,)) for i in range(self.workers)]
        t0 = time.perf_counter()
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        wall = time.perf_counter() - t0
        if errs or self._loop_err:
            raise RuntimeError(f"protocol run failed: {errs} {self._loop_err}")
        per_token = [max(bufs[i][t] for i in range(self.workers)) / 1e9 for t in range(tokens)]
        out = {"token_s": per_token, "wall_s": wall,
               "rounds": int(L.swl_wc_rounds(self.handles[0]))}
        if record:
            out["history"] = torch.cat(hist_c, 1)
        return out

    def close(self) -> None:
        L = lib()
        if self._loop is not None:
            extq.set_quit(1)
            self._loop.join(timeout=60)
            self._loop = None
        for h in self.handles:
            L.swl_wc_destroy(h)
        self.handles = []
        if getattr(self, "_queue_open", False):
            check(L.swl_agg_set_completion_mode(0))
            check(L.swl_agg_set_round_graphs(0))
            extq.close_queue()
            self._queue_open = False
