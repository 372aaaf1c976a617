"""One GPU's aggregator group stepped as a unit: the frozen base in the
aggregator's slot pool plus N worker slots, each with its own LoRA adapter,
RMSNorm weights and paged KV cache.

`SlotGroup.step()` enqueues one decode token for every slot — the per-token
loop of the reference's worker (worker_sync.py:1274-1425,
_generate_one_token_all) with the aggregator's 1 + 4*L + 1 rounds
(ext_aggregator.cpp:1095-1202) — as a fixed sequence of launches:

  tokens -> slot inputs, EMBED round, embeddings -> hidden
  per layer:
    RMSNorm(h) -> slot input          LoRA shrink (x @ A_qkv)
    QKV round (slot in -> slot out)   LoRA expand + add -> qkv
    RoPE + paged KV append            attention -> slot input
    LoRA shrink (attn @ A_o)          O round
    LoRA expand, + residual -> h      RMSNorm(h) -> slot input
    LoRA shrink (x @ A_gu)            Gate+Up round
    LoRA expand, SiLU*mul -> slot in  LoRA shrink (act @ A_down)
    Down round                        LoRA expand, + residual -> h
  RMSNorm(h) -> slot input, LM_HEAD round (greedy), next token -> tokens,
  KV positions += 1

Every launch reads/writes the slot buffers in place, so the sequence has no
host synchronisation and is captured once into a CUDA graph (`capture`) and
replayed per token. Rounds go through the aggregator's C-ABI round entry
(ownership and buffer bounds checked at capture time).
"""
from __future__ import annotations

import copy
import ctypes as C
import math
from dataclasses import dataclass, field

import torch

from . import ext_aggregator as agg
from . import worker_ops as wo
from ._native import check, i32_array, i64_array, lib, ptr_array

BF16 = torch.bfloat16


@dataclass
class ModelConfig:
    hidden: int = 4096
    inter: int = 14336
    layers: int = 32
    hq: int = 32
    hkv: int = 8
    head_dim: int = 128
    vocab: int = 128256
    rank: int = 16
    alpha: int = 32
    eps: float = 1e-5
    page: int = 16
    max_seq_per_step: int = 16
    rope_theta: float = 500000.0
    rope_scaling: dict = field(default_factory=lambda: {
        "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 8192, "rope_type": "llama3"})

    @property
    def qkv_n(self) -> int:
        return (self.hq + 2 * self.hkv) * self.head_dim


LLAMA_3_1_8B = ModelConfig()


def cos_sin_cache(cfg: ModelConfig, max_pos: int, device) -> torch.Tensor:
    """build_vllm_cos_sin_cache (paged_attention.py:131-142) from HF's
    LlamaRotaryEmbedding inv_freq (model_builder.py:293-303)."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    hf = LlamaConfig(hidden_size=cfg.hidden, num_attention_heads=cfg.hq,
                     num_key_value_heads=cfg.hkv, head_dim=cfg.head_dim,
                     rope_theta=cfg.rope_theta, rope_scaling=dict(cfg.rope_scaling) if cfg.rope_scaling else None,
                     max_position_embeddings=max(max_pos, 131072))
    inv = LlamaRotaryEmbedding(config=hf).inv_freq.float().cpu()
    t = torch.arange(max_pos, dtype=torch.float32)
    f = torch.outer(t, inv)
    return torch.cat([f.cos().to(BF16), f.sin().to(BF16)], -1).to(device)


@dataclass
class BaseWeights:
    """Frozen base model in HF layout ([out, in], bf16) on the device."""
    q: list
    k: list
    v: list
    o: list
    gate: list
    up: list
    down: list
    in_norm: list
    post_norm: list
    final_norm: torch.Tensor
    embed: torch.Tensor
    lm_head: torch.Tensor


def random_base(cfg: ModelConfig, seed: int, device, std: float = 0.02,
                norm_noise: float = 0.0) -> BaseWeights:
    """Seeded random-init base weights ~ N(0, std)."""
    g = torch.Generator(device=device).manual_seed(seed)

    def w(*shape):
        return (torch.randn(*shape, generator=g, device=device) * std).to(BF16)

    def norm():
        return (1.0 + norm_noise * torch.randn(cfg.hidden, generator=g, device=device)).to(BF16)

    H, I, D = cfg.hidden, cfg.inter, cfg.head_dim
    L = cfg.layers
    return BaseWeights(
        q=[w(cfg.hq * D, H) for _ in range(L)], k=[w(cfg.hkv * D, H) for _ in range(L)],
        v=[w(cfg.hkv * D, H) for _ in range(L)], o=[w(H, cfg.hq * D) for _ in range(L)],
        gate=[w(I, H) for _ in range(L)], up=[w(I, H) for _ in range(L)],
        down=[w(H, I) for _ in range(L)],
        in_norm=[norm() for _ in range(L)], post_norm=[norm() for _ in range(L)],
        final_norm=norm(), embed=w(cfg.vocab, H), lm_head=w(cfg.vocab, H))


def random_adapter(cfg: ModelConfig, seed: int, device, std: float = 0.02, rank: int | None = None) -> list:
    """Per layer: {'q': (A [r, in], B [out, r]), ...}, A, B ~ N(0, std); r is
    `rank` (default cfg.rank)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, I, D = cfg.hidden, cfg.inter, cfg.head_dim
    r = int(rank) if rank else cfg.rank
    dims = {"q": (H, cfg.hq * D), "k": (H, cfg.hkv * D), "v": (H, cfg.hkv * D),
            "o": (cfg.hq * D, H), "gate": (H, I), "up": (H, I), "down": (I, H)}
    out = []
    for _ in range(cfg.layers):
        layer = {}
        for name, (i, o) in dims.items():
            layer[name] = ((torch.randn(r, i, generator=g, device=device) * std).to(BF16),
                           (torch.randn(o, r, generator=g, device=device) * std).to(BF16))
        out.append(layer)
    return out


def exchange_with_peer(mine: bytes, rank: int, group=None) -> bytes:
    """Gives `mine` to the other rank of a two-rank torch.distributed group
    and returns what that rank gave (the IPC handles of the column-sharded
    variant)."""
    import torch.distributed as dist
    if dist.get_world_size(group) != 2 or rank not in (0, 1):
        raise ValueError("the peer exchange needs a group of exactly two ranks")
    both = [None, None]
    dist.all_gather_object(both, bytes(mine), group=group)
    return both[1 - rank]


class SlotGroup:
    """N decode slots on one aggregator (this process owns the pool)."""

    def __init__(self, cfg: ModelConfig, base: BaseWeights, adapters: list, ctx_lens: list,
                 max_new: int, device: int = 0, seed: int = 0, kv_std: float = 1.0,
                 round_algo: int = 0, worker_id0: int = 1000, fused: bool = True,
                 prefetch=(), prefetch_cap: int = 80 << 20, qkv_rope_fused: bool = False):
        self.cfg = cfg
        self.fused = fused
        if fused and cfg.hidden != 4096:
            raise ValueError(f"the fused step's RMSNorm epilogue is built for hidden 4096 (got {cfg.hidden}); "
                             "use fused=False for other sizes")
        # qkv_rope_fused: the QKV round carries the RoPE epilogue (one launch
        # instead of two; measured 3.5 us per layer slower than the separate
        # epilogue kernel at 28 slots, so off by default)
        self.qkv_rope_fused = bool(qkv_rope_fused) and "o" not in tuple(prefetch or ())
        self.prefetch = tuple(prefetch or ())
        self.pf_cap = int(prefetch_cap)
        self.dev = torch.device("cuda", device)
        self.n = n = len(ctx_lens)
        self.base = base
        H, I, D = cfg.hidden, cfg.inter, cfg.head_dim
        self.ctx0 = list(ctx_lens)
        self.max_len = max(ctx_lens) + max_new
        # --- aggregator: pool + fused weights ------------------------------------
        agg.init_slot_pool(n, device, H, I, cfg.hkv, D, cfg.max_seq_per_step, 2)
        agg.init_aggregator_begin(cfg.layers, device)
        for l in range(cfg.layers):
            agg.init_aggregator_layer(l, base.q[l], base.k[l], base.v[l], base.o[l],
                                      torch.empty(0), base.gate[l], base.up[l], base.down[l],
                                      torch.empty(0))
        agg.init_aggregator_finalize()
        agg.init_embed_lm_head_weights(base.embed, base.lm_head)
        agg.set_round_algo(round_algo)
        self.worker_ids = [worker_id0 + i for i in range(n)]
        self.slot_ids = [agg.claim_slot(w)["slot_id"] for w in self.worker_ids]
        bufs = [agg.slot_buffers(s) for s in self.slot_ids]
        self.slot_in = [b[0] for b in bufs]
        self.slot_out = [b[1] for b in bufs]
        # --- workers: adapters, KV, buffers ---------------------------------------
        # every adapter is packed at the group's rank cfg.rank (zero-padded
        # when smaller, its own alpha / r folded into the O / Down lora_B),
        # each slot's in one slab (a swap is one device copy)
        self.packed = [None if ad is None else
                       wo.pack_lora_slab(ad.layers, rank=ad.rank) if isinstance(ad, wo.PackedAdapter) else
                       self.pack_adapter(ad) for ad in adapters]
        self.lora = [None if p is None else p.layers for p in self.packed]
        pps = (self.max_len + cfg.page - 1) // cfg.page
        g = torch.Generator(device=self.dev).manual_seed(seed + 7)
        perm = torch.randperm(n * pps, generator=g, device=self.dev).to(torch.int32)
        self.block_tables = [perm[i * pps:(i + 1) * pps].contiguous() for i in range(n)]
        self.k_cache, self.v_cache = [], []
        for _ in range(cfg.layers):
            shape = (n * pps, cfg.page, cfg.hkv, D)
            self.k_cache.append((torch.randn(shape, generator=g, device=self.dev) * kv_std).to(BF16))
            self.v_cache.append((torch.randn(shape, generator=g, device=self.dev) * kv_std).to(BF16))
        self.seqlens = torch.tensor(ctx_lens, dtype=torch.int32, device=self.dev)
        self.cos_sin = cos_sin_cache(cfg, self.max_len + cfg.page, self.dev)
        # a step carries up to max_rows new tokens per slot (prefill chunks):
        # each slot's hidden rows are contiguous, h is every slot's first row
        self.max_rows = mr = int(cfg.max_seq_per_step)
        self.h_rows = torch.empty(n, mr, H, dtype=BF16, device=self.dev)
        self.h = self.h_rows[:, 0]
        self.qkv = torch.empty(n, cfg.qkv_n, dtype=BF16, device=self.dev)
        self.q_rot = torch.empty(n * mr, cfg.hq * D, dtype=BF16, device=self.dev)
        self.tok_in = torch.zeros(n, mr, dtype=torch.int64, device=self.dev)
        nparts = wo.attention_part_floats(n * mr, cfg.hq, cfg.hkv, self.max_len)
        self.part = torch.empty(max(1, nparts), dtype=torch.float32, device=self.dev)
        self.splits = max(1, min(8, -(-296 // n)))
        self.ws = torch.empty(self.splits * n * 3 * cfg.rank, dtype=torch.float32, device=self.dev)
        # fused path: LoRA shrink partials of each round's input, produced by the
        # epilogue kernel that writes that input
        self.norm_splits = int(lib().swl_fused_norm_splits(cfg.rank))
        self.dn_splits = int(lib().swl_fused_silu_splits(I))
        f32 = dict(dtype=torch.float32, device=self.dev)
        self.ws_qkv = torch.zeros(self.norm_splits * n * mr * 3 * cfg.rank, **f32)
        self.ws_o = torch.zeros(cfg.hq * n * mr * cfg.rank, **f32)
        self.ws_gu = torch.zeros(self.norm_splits * n * mr * 2 * cfg.rank, **f32)
        self.ws_dn = torch.zeros(self.dn_splits * n * mr * cfg.rank, **f32)
        self.tokens = torch.zeros(n, dtype=torch.int64, device=self.dev)
        self._build_call_args()
        self._advance = {}
        self._subset = None          # slot indices of a subset view (SlotGroup.subset), else None
        self._slot_index = list(range(n))
        self.graph = None

    # ------------------------------------------------------------------------------
    def _build_call_args(self):
        cfg, n = self.cfg, self.n
        H, I, D, r = cfg.hidden, cfg.inter, cfg.head_dim, cfg.rank
        self.a_rows = i32_array([1] * n)
        self.a_sids = i32_array(self.slot_ids)
        self.a_wids = i32_array(self.worker_ids)
        self.a_ones = i64_array([1] * n)
        self.a_in = ptr_array(self.slot_in)
        self.a_out = ptr_array(self.slot_out)
        self.a_h = ptr_array([self.h_rows[i].data_ptr() for i in range(n)])
        self.a_qkv = ptr_array([self.qkv[i].data_ptr() for i in range(n)])
        self.a_tok = ptr_array([self.tokens[i].data_ptr() for i in range(n)])
        self.a_b8 = i64_array([8] * n)
        self.a_bH = i64_array([2 * H] * n)
        self.a_bt = ptr_array([t.data_ptr() for t in self.block_tables])
        self.a_sl = ptr_array([self.seqlens[i].data_ptr() for i in range(n)])
        self.a_kc = [ptr_array([k.data_ptr()] * n) for k in self.k_cache]
        self.a_vc = [ptr_array([v.data_ptr()] * n) for v in self.v_cache]

        def per_layer(attr):
            return [ptr_array([None if self.lora[i] is None else
                               getattr(self.lora[i][l], attr).data_ptr() for i in range(n)])
                    for l in range(cfg.layers)]
        self.A_qkv, self.B_qkv = per_layer("A_qkv"), per_layer("B_qkv")
        self.A_o, self.B_o = per_layer("A_o"), per_layer("B_o")
        self.A_gu, self.B_gu = per_layer("A_gu"), per_layer("B_gu")
        self.A_dn, self.B_dn = per_layer("A_down"), per_layer("B_down")
        # next-round weights for the L2 prefetch issued by the worker kernels
        self.wptr = {}
        names = {agg.OP_QKV_FUSED: "qkv", agg.OP_O_PROJ: "o", agg.OP_GATE_UP_FUSED: "gate_up",
                 agg.OP_DOWN_PROJ: "down"}
        for l in range(cfg.layers):
            for op, nm in names.items():
                if nm not in self.prefetch:
                    continue
                W, N_, K_ = C.c_void_p(), C.c_int64(), C.c_int64()
                check(lib().swl_agg_weight(l, op, C.byref(W), C.byref(N_), C.byref(K_)))
                self.wptr[(l, op)] = (W.value, min(2 * N_.value * K_.value, self.pf_cap))
        if "lm_head" in self.prefetch:
            self.wptr["lm_head"] = (self.base.lm_head.data_ptr(),
                                    min(self.base.lm_head.numel() * 2, self.pf_cap))
        self.ends_qkv = i64_array([cfg.hq * D, (cfg.hq + cfg.hkv) * D, cfg.qkv_n])
        self.ends_gu = i64_array([I, 2 * I, 2 * I])
        self.ends_h = i64_array([H, H, H])
        self.scaling = cfg.alpha / r

    def pack_adapter(self, adapter, scaling: float | None = None) -> wo.PackedAdapter:
        """An adapter (per-layer dicts as random_adapter or
        adapters.AdapterLoader.load make, any rank up to the group's) packed
        at the group's rank into one slab: the form a cache of resident
        adapters keeps, ready for set_adapter. `scaling` is the adapter's
        lora_alpha / r (default the group's alpha / r); its ratio to the
        group's alpha / rank is folded into the O / Down lora_B, exact when
        that ratio is a power of two."""
        cfg = self.cfg
        r = int(adapter[0]["q"][0].shape[0])
        if not 1 <= r <= cfg.rank:
            raise ValueError(f"adapter rank {r}: must be at most the group's rank {cfg.rank}")
        s = float(scaling) if scaling is not None else cfg.alpha / r
        return wo.pack_lora_slab([wo.pack_lora_layer(adapter[l], s, pad_rank=cfg.rank,
                                                     post_scale=cfg.alpha / cfg.rank)
                                  for l in range(cfg.layers)], rank=r)

    def set_adapter(self, i: int, adapter) -> None:
        """Replaces slot i's adapter in place, from a PackedAdapter
        (pack_adapter: one device copy of its slab) or from per-layer dicts
        (packed first). The copy runs on the current stream into the slot's
        existing buffers, so a captured step graph keeps working and its next
        replay uses the new adapter. Call it between steps, ordered after the
        last step on that stream. A slot built without an adapter has no
        buffers to swap into."""
        if self.packed[i] is None:
            raise ValueError(f"slot {i} was built without an adapter")
        if not isinstance(adapter, wo.PackedAdapter):
            adapter = self.pack_adapter(adapter)
        dst = self.packed[i]
        if adapter.slab.numel() != dst.slab.numel() or adapter.slab.device != dst.slab.device:
            raise ValueError("packed adapter does not match the group's layout (model, rank or device)")
        dst.slab.copy_(adapter.slab)
        dst.rank = adapter.rank

    def _round(self, op, layer, st, tx=None):
        check(lib().swl_agg_execute_round(op, layer, self.n, self.a_sids, self.a_wids, self.a_ones,
                                          tx if tx is not None else self.a_ones, st))

    def enqueue_step(self, stream: torch.cuda.Stream, rows=None, tokens=None) -> None:
        """Queues one step on `stream` (no host sync). By default every slot
        decodes one token (its last output, `tokens`). With `rows` (new tokens
        per slot, 1..max_rows) and `tokens` (their ids, one list per slot) the
        step carries prefill chunks next to decode rows, the mixed
        configuration: every new row goes through the layers, its K / V is
        appended, and each slot's next token comes from its last row. A
        slot's entry of `tokens` may be None when it has one row: that row is
        the slot's last output, taken on the device (no host round trip).
        The ids are copied to the device first, so such a step is not for
        capture (see `capture(rows=...)`)."""
        if rows is None:
            if self.fused:
                return self._enqueue_fused(stream)
            return self._enqueue_unfused(stream)
        return self._enqueue_fused(stream, self._stage_tokens(stream, rows, tokens))

    def _stage_tokens(self, stream, rows, tokens) -> list:
        """Checks a mixed step's rows / tokens and copies the ids into tok_in
        (None: the slot's last output, on the device); returns the rows."""
        if not self.fused:
            raise ValueError("steps with several rows per slot run the fused sequence")
        rows = [int(x) for x in rows]
        if len(rows) != self.n or any(x < 1 or x > self.max_rows for x in rows):
            raise ValueError(f"rows: one count per slot in 1..{self.max_rows}")
        if tokens is None or len(tokens) != self.n or any(
                (t is None and x != 1) or (t is not None and len(t) != x) for t, x in zip(tokens, rows)):
            raise ValueError("tokens: one list of ids per slot, as long as its row count (None: one row, "
                             "the slot's last output)")
        with torch.cuda.stream(stream):
            if any(t is None for t in tokens):
                self.tok_in[:, 0].copy_(self.tokens)
            for j, (i, t) in enumerate(zip(self._slot_index, tokens)):
                if t is not None:
                    self.tok_in[i, :rows[j]].copy_(torch.tensor(t, dtype=torch.int64))
        return rows

    def _enqueue_fused(self, stream: torch.cuda.Stream, row_counts=None, mark=None) -> None:
        """Fused sequence: per layer 4 rounds + 6 worker kernels (each worker
        kernel finishes one round's epilogue and starts the next round's LoRA).
        mark(kind), when given, is called after each launch (profile_step)."""
        L, cfg, n, st = lib(), self.cfg, self.n, stream.cuda_stream
        mark = mark or (lambda kind: None)
        H, I, D, r = cfg.hidden, cfg.inter, cfg.head_dim, cfg.rank
        s = self.scaling
        nl = cfg.layers
        if row_counts is None:
            rows, tx = self.a_rows, None
            check(L.swl_copy_rows(n, self.a_tok, self.a_in, self.a_b8, st))
        else:
            rows, tx = i32_array(row_counts), i64_array(row_counts)
            check(L.swl_copy_rows(n, ptr_array([self.tok_in[i].data_ptr() for i in self._slot_index]), self.a_in,
                                  i64_array([8 * x for x in row_counts]), st))
        self._round(agg.OP_EMBED, 0, st, tx)
        mark("embed")
        # embedding -> h, RMSNorm -> QKV slot input, QKV shrink
        pf = self.wptr
        none = (None, 0)
        check(L.swl_fused_resid_norm_shrink(n, rows, self.a_out, H, None, 0, 0.0, None, 0, 0, self.a_h, H,
                                            self.base.in_norm[0].data_ptr(), H, cfg.eps, self.a_in, H,
                                            self.A_qkv[0], 3 * r, self.ws_qkv.data_ptr(),
                                            *pf.get((0, agg.OP_QKV_FUSED), none), st))
        mark("epilogue")
        for l in range(nl):
            if self.qkv_rope_fused:
                # the QKV round with the RoPE epilogue in its own epilogue
                check(L.swl_agg_execute_qkv_rope_round(l, n, self.a_sids, self.a_wids, self.a_ones,
                                                       tx if tx is not None else self.a_ones,
                                                       self.B_qkv[l], r, self.ws_qkv.data_ptr(), self.norm_splits,
                                                       self.a_bt, self.a_kc[l], self.a_vc[l], self.a_sl, cfg.hq,
                                                       cfg.hkv, D, cfg.page, self.cos_sin.data_ptr(),
                                                       self.q_rot.data_ptr(), st))
                mark("round")
            else:
                self._round(agg.OP_QKV_FUSED, l, st, tx)
                mark("round")
                check(L.swl_fused_qkv_rope(n, rows, self.a_out, cfg.qkv_n, self.B_qkv[l], r,
                                           self.ws_qkv.data_ptr(), self.norm_splits, self.a_bt, self.a_kc[l],
                                           self.a_vc[l], self.a_sl, cfg.hq, cfg.hkv, D, cfg.page,
                                           self.cos_sin.data_ptr(), self.q_rot.data_ptr(),
                                           *pf.get((l, agg.OP_O_PROJ), none), st))
                mark("epilogue")
            check(L.swl_paged_attention_shrink(n, rows, self.a_bt, self.a_kc[l], self.a_vc[l], self.a_sl,
                                               self.a_in, cfg.hq * D, cfg.hq, cfg.hkv, D, cfg.page,
                                               1.0 / math.sqrt(D), self.max_len, self.q_rot.data_ptr(),
                                               self.part.data_ptr(), self.A_o[l], r, self.ws_o.data_ptr(),
                                               None, 0, st))
            mark("attention")
            self._round(agg.OP_O_PROJ, l, st, tx)
            mark("round")
            check(L.swl_fused_resid_norm_shrink(n, rows, self.a_out, H, self.B_o[l], r, s, self.ws_o.data_ptr(),
                                                cfg.hq, 1, self.a_h, H, self.base.post_norm[l].data_ptr(), H,
                                                cfg.eps, self.a_in, H, self.A_gu[l], 2 * r,
                                                self.ws_gu.data_ptr(), *pf.get((l, agg.OP_GATE_UP_FUSED), none),
                                                st))
            mark("epilogue")
            self._round(agg.OP_GATE_UP_FUSED, l, st, tx)
            mark("round")
            check(L.swl_fused_gu_silu_shrink(n, rows, self.a_out, 2 * I, self.B_gu[l], r, self.ws_gu.data_ptr(),
                                             self.norm_splits, I, self.a_in, I, self.A_dn[l], r,
                                             self.ws_dn.data_ptr(), *pf.get((l, agg.OP_DOWN_PROJ), none), st))
            mark("epilogue")
            self._round(agg.OP_DOWN_PROJ, l, st, tx)
            mark("round")
            last = l == nl - 1
            w_next = self.base.final_norm if last else self.base.in_norm[l + 1]
            check(L.swl_fused_resid_norm_shrink(n, rows, self.a_out, H, self.B_dn[l], r, s, self.ws_dn.data_ptr(),
                                                self.dn_splits, 1, self.a_h, H, w_next.data_ptr(), H, cfg.eps,
                                                self.a_in, H, None if last else self.A_qkv[l + 1], 3 * r,
                                                self.ws_qkv.data_ptr(),
                                                *pf.get("lm_head" if last else (l + 1, agg.OP_QKV_FUSED), none),
                                                st))
            mark("epilogue")
        self._round(agg.OP_LM_HEAD, 0, st, tx)  # the greedy pick reads each slot's last row
        mark("lm_head")
        check(L.swl_copy_rows(n, self.a_out, self.a_tok, self.a_b8, st))
        if self._subset is None and (row_counts is None or len(set(row_counts)) == 1):
            check(L.swl_advance_i32(self.seqlens.data_ptr(), n, 1 if row_counts is None else row_counts[0], st))
        else:
            with torch.cuda.stream(stream):
                self.seqlens.add_(self._advance_of(self._full_pattern(row_counts)))

    def _full_pattern(self, row_counts) -> list:
        """Per-slot position advance over the whole group (0 outside a subset)."""
        rows = [1] * self.n if row_counts is None else [int(x) for x in row_counts]
        if self._subset is None:
            return rows
        full = [0] * len(self.slot_ids)
        for i, x in zip(self._subset, rows):
            full[i] = x
        return full

    def _advance_of(self, row_counts, keep: bool = False) -> torch.Tensor:
        """Device copy of a row pattern (the per-slot position advance). A
        captured graph reads its copy on every replay, so `capture` makes it
        beforehand and keeps it (keep=True); an eager step uses a temporary
        (its memory returns to the stream's pool once the add has run)."""
        key = tuple(int(x) for x in row_counts)
        t = self._advance.get(key)
        if t is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("a new row pattern inside a graph capture: pass it to capture(rows=...)")
            t = torch.tensor(key, dtype=torch.int32, device=self.dev)
            if keep:
                self._advance[key] = t
        return t

    def _enqueue_unfused(self, stream: torch.cuda.Stream) -> None:
        """Modular sequence (one kernel per operation), kept as a cross-check."""
        L, cfg, n, st = lib(), self.cfg, self.n, stream.cuda_stream
        H, I, D, r = cfg.hidden, cfg.inter, cfg.head_dim, cfg.rank
        sp, ws = self.splits, self.ws.data_ptr()
        rows = self.a_rows
        check(L.swl_copy_rows(n, self.a_tok, self.a_in, self.a_b8, st))
        self._round(agg.OP_EMBED, 0, st)
        check(L.swl_copy_rows(n, self.a_out, self.a_h, self.a_bH, st))
        for l in range(cfg.layers):
            check(L.swl_rms_norm(n, rows, self.a_h, H, self.a_in, H, self.base.in_norm[l].data_ptr(),
                                 H, cfg.eps, st))
            check(L.swl_lora_shrink(n, rows, self.a_in, H, self.A_qkv[l], H, 3 * r, sp, ws, st))
            self._round(agg.OP_QKV_FUSED, l, st)
            check(L.swl_lora_expand(n, rows, self.a_out, cfg.qkv_n, self.B_qkv[l], None, 0, self.a_qkv,
                                    cfg.qkv_n, cfg.qkv_n, r, 3, self.ends_qkv, 0.0, wo.EXPAND_ADD, sp,
                                    ws, st))
            check(L.swl_rope_append(n, rows, self.a_qkv, cfg.qkv_n, self.a_bt, self.a_kc[l],
                                    self.a_vc[l], self.a_sl, cfg.hq, cfg.hkv, D, cfg.page,
                                    self.cos_sin.data_ptr(), self.cos_sin.shape[0],
                                    self.q_rot.data_ptr(), st))
            check(L.swl_paged_attention(n, rows, self.a_bt, self.a_kc[l], self.a_vc[l], self.a_sl,
                                        self.a_in, cfg.hq * D, cfg.hq, cfg.hkv, D, cfg.page,
                                        1.0 / math.sqrt(D), self.max_len, self.q_rot.data_ptr(),
                                        self.part.data_ptr(), st))
            check(L.swl_lora_shrink(n, rows, self.a_in, cfg.hq * D, self.A_o[l], cfg.hq * D, r, sp,
                                    ws, st))
            self._round(agg.OP_O_PROJ, l, st)
            check(L.swl_lora_expand(n, rows, self.a_out, H, self.B_o[l], self.a_h, H, self.a_h, H, H,
                                    r, 1, self.ends_h, self.scaling, wo.EXPAND_RESIDUAL, sp, ws, st))
            check(L.swl_rms_norm(n, rows, self.a_h, H, self.a_in, H, self.base.post_norm[l].data_ptr(),
                                 H, cfg.eps, st))
            check(L.swl_lora_shrink(n, rows, self.a_in, H, self.A_gu[l], H, 2 * r, sp, ws, st))
            self._round(agg.OP_GATE_UP_FUSED, l, st)
            check(L.swl_lora_expand(n, rows, self.a_out, 2 * I, self.B_gu[l], None, 0, self.a_in, I,
                                    2 * I, r, 2, self.ends_gu, 0.0, wo.EXPAND_SILU_MUL, sp, ws, st))
            check(L.swl_lora_shrink(n, rows, self.a_in, I, self.A_dn[l], I, r, sp, ws, st))
            self._round(agg.OP_DOWN_PROJ, l, st)
            check(L.swl_lora_expand(n, rows, self.a_out, H, self.B_dn[l], self.a_h, H, self.a_h, H, H,
                                    r, 1, self.ends_h, self.scaling, wo.EXPAND_RESIDUAL, sp, ws, st))
        check(L.swl_rms_norm(n, rows, self.a_h, H, self.a_in, H, self.base.final_norm.data_ptr(), H,
                             cfg.eps, st))
        self._round(agg.OP_LM_HEAD, 0, st)
        check(L.swl_copy_rows(n, self.a_out, self.a_tok, self.a_b8, st))
        check(L.swl_advance_i32(self.seqlens.data_ptr(), n, 1, st))

    def profile_step(self, stream: torch.cuda.Stream | None = None, rows=None, tokens=None,
                     print_line: bool | None = None) -> dict:
        """Runs one step eagerly with a CUDA event after every launch and
        returns the device time per launch kind in microseconds (embed,
        round, attention, epilogue, lm_head) and the step's wall time, as the
        reference worker's profiled token does (worker_sync.py:1427-1782,
        PROFILE_LAYERS=1). Prints the reference's `[LAYER_PROFILE]` line
        (gather_us / scatter_us are 0: rounds read and write the slot buffers
        in place) when print_line is True, or None and PROFILE_LAYERS=1. The
        events end programmatic overlap between launches, so the sum is an
        upper bound of a replayed step."""
        import os
        import time
        if not self.fused:
            raise ValueError("profile_step runs the fused sequence")
        s = stream or torch.cuda.current_stream(self.dev)
        events = []

        def mark(kind):
            e = torch.cuda.Event(enable_timing=True)
            e.record(s)
            events.append((kind, e))
        torch.cuda.synchronize(self.dev)
        t0 = time.perf_counter()
        start = torch.cuda.Event(enable_timing=True)
        start.record(s)
        if rows is None:
            self._enqueue_fused(s, mark=mark)
        else:
            self._enqueue_fused(s, self._stage_tokens(s, rows, tokens), mark=mark)
        end = torch.cuda.Event(enable_timing=True)
        end.record(s)
        end.synchronize()
        wall_us = (time.perf_counter() - t0) * 1e6
        out = {k: 0.0 for k in ("embed", "round", "attention", "epilogue", "lm_head")}
        prev = start
        for kind, e in events:
            out[kind] += prev.elapsed_time(e) * 1e3
            prev = e
        out["device_us"] = start.elapsed_time(end) * 1e3
        out["wall_us"] = wall_us
        self._profile_token = getattr(self, "_profile_token", 0) + 1
        if print_line or (print_line is None and os.environ.get("PROFILE_LAYERS") == "1"):
            wid = self.worker_ids[self._slot_index[0]]
            compute = wall_us  # no gather / scatter copies
            print(f"[LAYER_PROFILE] worker={wid} token={self._profile_token} gather_us=0 scatter_us=0 "
                  f"compute_us={compute:.0f} wall_us={wall_us:.0f} ipc_pct=0.0 slots={self.n} "
                  f"round_us={out['round']:.0f} attn_us={out['attention']:.0f} epi_us={out['epilogue']:.0f} "
                  f"embed_us={out['embed']:.0f} lm_head_us={out['lm_head']:.0f} device_us={out['device_us']:.0f}",
                  flush=True)
        return out

    def launches_per_step(self) -> int:
        """Kernel launches of one step of this library's kernels."""
        if self.fused:
            # copy, embed, embed-norm; per layer 4 rounds + qkv_rope (unless the QKV round carries it)
            # + attention (2) + 3 epilogues; LM head GEMM + argmax, copy, advance
            per_layer = 9 if self.qkv_rope_fused else 10
            return 3 + self.cfg.layers * per_layer + 2 + 2
        per_layer = 2 + 4 * 3 + 1 + 2  # norms, (shrink+round+expand)x4, rope, attention + combine
        return 3 + self.cfg.layers * per_layer + 1 + 2 + 1 + 1

    def capture(self, stream: torch.cuda.Stream | None = None, rows=None) -> None:
        """Captures one step into a CUDA graph (replayed by `replay`). Capture
        does not execute the step, so the state is unchanged. With `rows`
        (new tokens per slot, a fixed mixed pattern) the graph reads each
        slot's token ids from `tok_in[i, :rows[i]]`, which the caller fills
        before every replay."""
        s = stream or torch.cuda.Stream(self.dev)
        if rows is not None:
            rows = [int(x) for x in rows]
            if len(rows) != self.n or any(x < 1 or x > self.max_rows for x in rows) or not self.fused:
                raise ValueError(f"rows: one count per slot in 1..{self.max_rows} (fused sequence)")
        if self._subset is not None or (rows is not None and len(set(rows)) > 1):
            self._advance_of(self._full_pattern(rows), keep=True)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            if rows is None:
                self.enqueue_step(s)
            else:
                self._enqueue_fused(s, rows)

    def replay(self) -> None:
        self.graph.replay()

    def read_slot_rows(self, which: str, row_elems: int, dtype=BF16) -> torch.Tensor:
        """Copies row 0 of every slot's input ('in') or output ('out') buffer
        into a [n, row_elems] tensor (for checks; synchronises)."""
        out = torch.empty(self.n, row_elems, dtype=dtype, device=self.dev)
        src = self.a_in if which == "in" else self.a_out
        nbytes = row_elems * out.element_size()
        check(lib().swl_copy_rows(self.n, src, ptr_array([out[i].data_ptr() for i in range(self.n)]),
                                  i64_array([nbytes] * self.n), torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        return out

    def set_context(self, i: int, length: int = 0) -> None:
        """Sets slot i's cached length (a new request starts at 0; its pages
        are reused), ordered on the current stream."""
        if not 0 <= length <= self.max_len:
            raise ValueError(f"context {length} outside 0..{self.max_len}")
        self.seqlens[i].fill_(int(length))

    def reset_positions(self) -> None:
        self.seqlens.copy_(torch.tensor(self.ctx0, dtype=torch.int32))

    def shard(self, rank: int, group=None) -> None:
        """Column-sharded base weights with the other GPU of a two-process
        torch.distributed `group` (both processes built with the same seeds
        and inputs): from here on every round computes this GPU's half of the
        output columns and writes it into both GPUs' slot outputs; the
        worker-side kernels run on both GPUs. Call before `capture`."""
        import torch.distributed as dist
        agg.shard_begin(rank, 2)
        agg.shard_connect(exchange_with_peer(agg.shard_handles(), rank, group))
        dist.barrier(group=group)
        self._shard_group = (group,)

    def subset(self, active) -> "SlotGroup":
        """A view of this group whose steps run only the slots in `active`
        (indices into this group): adapters, caches, positions and buffers
        are shared, the kernels and rounds see only those slots (an idle
        slot costs nothing, not even its adapter's bytes), positions advance
        for those slots only, and the view keeps its own CUDA graph
        (`capture` / `replay`). Its `rows` / `tokens` arguments have one
        entry per active slot, in `active` order; `set_context` and
        `set_adapter` still take group indices. Closing the view only drops
        its graph; a view (and its graph) is usable only while its group is
        open, since it launches on the group's buffers."""
        if self._subset is not None:
            raise ValueError("a subset of a subset view")
        if not self.fused:
            raise ValueError("subset views run the fused sequence")
        active = sorted(set(int(i) for i in active))
        if not active or active[0] < 0 or active[-1] >= self.n:
            raise ValueError(f"active slots must be indices in 0..{self.n - 1}")
        v = copy.copy(self)
        v._subset, v._slot_index, v.n, v.graph = tuple(active), list(active), len(active), None

        def ptrs(arr):
            return ptr_array([arr[i] for i in active])
        k = len(active)
        v.a_rows, v.a_ones = i32_array([1] * k), i64_array([1] * k)
        v.a_sids = i32_array([self.slot_ids[i] for i in active])
        v.a_wids = i32_array([self.worker_ids[i] for i in active])
        v.a_in, v.a_out, v.a_h, v.a_qkv = ptrs(self.a_in), ptrs(self.a_out), ptrs(self.a_h), ptrs(self.a_qkv)
        v.a_tok, v.a_bt, v.a_sl = ptrs(self.a_tok), ptrs(self.a_bt), ptrs(self.a_sl)
        v.a_b8, v.a_bH = i64_array([8] * k), i64_array([2 * self.cfg.hidden] * k)
        v.a_kc = [ptr_array([t.data_ptr()] * k) for t in self.k_cache]
        v.a_vc = [ptr_array([t.data_ptr()] * k) for t in self.v_cache]
        for name in ("A_qkv", "B_qkv", "A_o", "B_o", "A_gu", "B_gu", "A_dn", "B_dn"):
            setattr(v, name, [ptrs(t) for t in getattr(self, name)])
        return v

    def close(self) -> None:
        self.graph = None
        if self._subset is not None:
            return
        if getattr(self, "_shard_group", None) is not None:
            import torch.distributed as dist
            torch.cuda.synchronize(self.dev)
            agg.shard_end()
            dist.barrier(group=self._shard_group[0])  # neither frees its pool while the peer maps it
            self._shard_group = None
        for s, w in zip(self.slot_ids, self.worker_ids):
            agg.release_slot(s, w)
        agg.cleanup_slot_pool()
