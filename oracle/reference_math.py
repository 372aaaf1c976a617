"""CPU restatement of the reference's hot-path arithmetic (test infrastructure).

Conventions: inputs and outputs are bf16 CPU tensors; every matmul runs in
fp32 and is rounded to bf16 where the reference's torch/cuBLAS call returns a
bf16 tensor; elementwise bf16 ops are restated as fp32 op + bf16 rounding,
which is what torch's bf16 kernels do per operation.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

BF16 = torch.bfloat16


def bf(x: torch.Tensor) -> torch.Tensor:
    return x.to(BF16)


def mm_bf16(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a @ b for bf16 operands with fp32 accumulation and a bf16 result."""
    return bf(a.float() @ b.float())


# ---------------------------------------------------------------------------
# Aggregator round: ext_aggregator.cpp:470-626
# ---------------------------------------------------------------------------

def fuse_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """ext_aggregator.cpp:366-367: cat(q, k, v) along the output dimension."""
    return torch.cat([q, k, v], 0)


def fuse_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """ext_aggregator.cpp:369-370: cat(gate, up) along the output dimension."""
    return torch.cat([gate, up], 0)


def slot_round(inputs: list[torch.Tensor], W: torch.Tensor,
               bias: torch.Tensor | None = None) -> list[torch.Tensor]:
    """One gather -> GEMM -> scatter round (ext_aggregator.cpp:526-625).

    inputs[i] is slot i's [rows_i, K] activation. The reference concatenates
    them (torch::cat, :551), runs matmul_out(out, x_flat, W.t()) into a bf16
    staging buffer (:562/:576/:598/:612), adds a non-empty bias in bf16
    (:580/:616) and copies each slot's rows back (:564-570).
    """
    rows = [int(x.shape[0]) for x in inputs]
    x = torch.cat(inputs, 0)
    y = mm_bf16(x, W.t())
    if bias is not None and bias.numel() > 0:
        y = bf(y.float() + bias.float())
    return list(torch.split(y, rows, 0))


def embed_round(token_lists: list[torch.Tensor], table: torch.Tensor) -> list[torch.Tensor]:
    """ext_aggregator.cpp:669-705: clamp ids to [0, vocab) and gather rows."""
    out = []
    for ids in token_lists:
        ids = ids.reshape(-1).long().clamp(0, table.shape[0] - 1)
        out.append(table[ids])
    return out


def lm_head_logits(last_hidden: torch.Tensor, W_lm: torch.Tensor) -> torch.Tensor:
    """ext_aggregator.cpp:818-821: logits = last_hidden @ W_lm^T (bf16)."""
    return mm_bf16(last_hidden, W_lm.t())


def greedy(logits: torch.Tensor) -> torch.Tensor:
    """ext_aggregator.cpp:859-861: argmax (first maximal index)."""
    return logits.float().argmax(-1)


def sample_distribution(logits: torch.Tensor, temperature: float, top_k: int,
                        top_p: float) -> tuple[torch.Tensor, float]:
    """The distribution the LM head samples one row of bf16 logits from
    (ext_aggregator.cpp:757-787, :821-861): logits * (1 / max(T, 0.01))
    rounded to bf16 (torch's bf16 division by a scalar multiplies by the
    reciprocal), the top_k largest kept (ties at the k-th value kept:
    `logits < threshold -> -inf`), then in descending order (ties in index
    order) the tokens whose running probability is <= top_p, the first
    always, then the softmax. The running sums are exact (float64) where the
    reference rounds them to bf16. Returns (probabilities [V] float64, margin):
    margin is the distance of top_p from the nearest running sum (inf without
    top-p), i.e. how far the cut is from flipping."""
    x = logits.reshape(-1)
    V = x.numel()
    inv = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(max(float(temperature), 0.01), dtype=torch.float32)
    xf = bf(x.float() * inv).double()
    neg = torch.tensor(-math.inf, dtype=torch.float64)
    keep = ~torch.isnan(xf)
    if 0 < top_k < V:
        thr = torch.topk(torch.where(keep, xf, neg), top_k).values[-1]
        keep &= xf >= thr
    xm = xf[keep].max()
    w = torch.where(keep, torch.exp(xf - xm), torch.zeros((), dtype=torch.float64))
    margin = math.inf
    if top_p < 1.0:
        order = torch.sort(torch.where(keep, xf, neg), descending=True, stable=True).indices
        order = order[keep[order]]
        cum = torch.cumsum(w[order], 0) / w.sum()
        stay = cum <= top_p
        stay[0] = True
        margin = float((cum - top_p).abs().min())
        cut = torch.zeros(V, dtype=torch.bool)
        cut[order[stay]] = True
        w = torch.where(cut, w, torch.zeros((), dtype=torch.float64))
    return w / w.sum(), margin


def sample_allowed(logits: torch.Tensor, temperature: float, top_k: int, top_p: float,
                   slack: float) -> torch.Tensor:
    """Tokens a correct sampler may draw from for one row when its running
    sums carry rounding: the kept set of sample_distribution plus the tokens
    whose exact running probability lies within `slack` above top_p."""
    probs, _ = sample_distribution(logits, temperature, top_k, top_p + slack if top_p < 1.0 else top_p)
    return probs > 0


def sample_token(logits: torch.Tensor, do_sample: bool, temperature: float, top_k: int, top_p: float,
                 u: float) -> tuple[int, float]:
    """The LM head's next token for one row: the argmax (greedy), or the
    draw from sample_distribution restated as the inverse CDF in index order
    at the uniform u (the reference's torch.multinomial stream is not
    reproducible; its distribution is). Returns (token, margin): the
    distance of u and of top_p from the nearest decision boundary."""
    x = logits.reshape(-1)
    if not do_sample:
        return int(x.float().argmax()), math.inf
    probs, margin = sample_distribution(x, temperature, top_k, top_p)
    cdf = torch.cumsum(probs, 0)
    kept_idx = (probs > 0).nonzero().flatten()
    token = int(torch.searchsorted(cdf, torch.tensor([float(u)], dtype=torch.float64), right=True)[0])
    token = min(token, int(kept_idx[-1]))
    margin = min(margin, float((cdf[kept_idx] - float(u)).abs().min()))
    return token, margin


# ---------------------------------------------------------------------------
# Worker LoRA: model_builder.py:217-262, worker_sync.py:305/:375
# ---------------------------------------------------------------------------

def pack_fused_lora(As: list[torch.Tensor], Bs: list[torch.Tensor], scaling: float,
                    out_dims: list[int]) -> tuple[torch.Tensor, torch.Tensor]:
    """FusedLoRA.__init__ (model_builder.py:231-255).

    A' = cat_i(A_i^T * s) [in, n*r] with the scale applied in bf16, and B' the
    block-diagonal [n*r, sum(out_dims)] holding B_i^T in block i.
    """
    A_cols = [bf(A.t().float() * scaling) for A in As]
    fused_A = torch.cat(A_cols, 1)
    r = As[0].shape[0]
    fused_B = torch.zeros(r * len(Bs), sum(out_dims), dtype=BF16)
    col = 0
    for i, B in enumerate(Bs):
        fused_B[i * r:(i + 1) * r, col:col + out_dims[i]] = B.t()
        col += out_dims[i]
    return fused_A, fused_B


def fused_lora_delta(x: torch.Tensor, fused_A: torch.Tensor, fused_B: torch.Tensor,
                     out_dims: list[int]) -> list[torch.Tensor]:
    """FusedLoRA.forward (model_builder.py:258-262): (x @ A') @ B', split."""
    t = mm_bf16(x, fused_A)
    d = mm_bf16(t, fused_B)
    return list(torch.split(d, out_dims, -1))


def lora_delta_scale_after(x: torch.Tensor, A: torch.Tensor, B: torch.Tensor,
                           scaling: float) -> torch.Tensor:
    """O / Down LoRA (worker_sync.py:305, :375): lora_B(lora_A(x)) * scaling."""
    t = mm_bf16(x, A.t())
    d = mm_bf16(t, B.t())
    return bf(d.float() * scaling)


def add_bf16(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return bf(a.float() + b.float())


# ---------------------------------------------------------------------------
# Norm / activation (HF LlamaRMSNorm, worker_sync.py:151-158)
# ---------------------------------------------------------------------------

def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """LlamaRMSNorm: fp32 normalise, round to bf16, times the bf16 weight."""
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return bf(w.float() * bf(h).float())


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """F.silu(gate) * up in bf16 (two rounded bf16 ops)."""
    g = gate.float()
    s = bf(g / (1.0 + torch.exp(-g)))
    return bf(s.float() * up.float())


# ---------------------------------------------------------------------------
# RoPE: paged_attention.py:131-142 + vLLM rotary_embedding(is_neox=True)
# ---------------------------------------------------------------------------

def llama3_inv_freq(head_dim: int = 128, theta: float = 500000.0, factor: float = 8.0,
                    low_freq_factor: float = 1.0, high_freq_factor: float = 4.0,
                    original_max_pos: int = 8192) -> torch.Tensor:
    """inv_freq of HF LlamaRotaryEmbedding for rope_type "llama3" (Llama-3.1)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    low_wl = original_max_pos / low_freq_factor
    high_wl = original_max_pos / high_freq_factor
    wavelen = 2 * math.pi / inv
    inv_l = torch.where(wavelen > low_wl, inv / factor, inv)
    smooth = (original_max_pos / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
    smoothed = (1 - smooth) * inv_l / factor + smooth * inv_l
    is_medium = ~(wavelen < high_wl) * ~(wavelen > low_wl)
    return torch.where(is_medium, smoothed, inv_l)


def cos_sin_cache(inv_freq: torch.Tensor, max_seq_len: int) -> torch.Tensor:
    """build_vllm_cos_sin_cache (paged_attention.py:131-142): [max_seq, D] = cos|sin in bf16."""
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq.float())
    return torch.cat([bf(freqs.cos()), bf(freqs.sin())], -1)


def rope_neox(x: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor,
              head_dim: int) -> torch.Tensor:
    """vLLM rotary_embedding, NeoX layout, bf16 arithmetic per op.

    x: [T, n_heads * head_dim]. For each head, with half = head_dim / 2,
    x1 = x[:half], x2 = x[half:], c/s from cache[pos]:
    out1 = bf(bf(x1*c) - bf(x2*s)), out2 = bf(bf(x2*c) + bf(x1*s)).
    """
    T = x.shape[0]
    h = x.reshape(T, -1, head_dim).float()
    half = head_dim // 2
    cs = cache[positions.long()].float()  # [T, D]
    c = cs[:, None, :half]
    s = cs[:, None, half:]
    x1, x2 = h[..., :half], h[..., half:]
    o1 = bf(bf(x1 * c).float() - bf(x2 * s).float())
    o2 = bf(bf(x2 * c).float() + bf(x1 * s).float())
    return torch.cat([o1, o2], -1).reshape(T, -1)


# ---------------------------------------------------------------------------
# Paged KV + attention: paged_attention.py:7-128, flash_attn_with_kvcache
# ---------------------------------------------------------------------------

@dataclass
class PagedKV:
    """Block bookkeeping of PagedKVCache (paged_attention.py:7-128) for one
    layer set; caches are [num_blocks, block, kv_heads, head_dim] bf16."""
    num_layers: int
    num_blocks: int
    block_size: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    k: list = field(default_factory=list)
    v: list = field(default_factory=list)
    free: list = field(default_factory=list)
    tables: dict = field(default_factory=dict)
    seq_lens: dict = field(default_factory=dict)

    def __post_init__(self):
        shape = (self.num_blocks, self.block_size, self.kv_heads, self.head_dim)
        self.k = [torch.zeros(shape, dtype=BF16) for _ in range(self.num_layers)]
        self.v = [torch.zeros(shape, dtype=BF16) for _ in range(self.num_layers)]
        self.free = list(range(self.num_blocks - 1, -1, -1))

    def ensure(self, slot: int, needed_len: int) -> None:
        """ensure_blocks_for_length / allocate_blocks (:57-75)."""
        need = (needed_len + self.block_size - 1) // self.block_size
        have = len(self.tables.get(slot, []))
        if need > have:
            if len(self.free) < need - have:
                raise RuntimeError("PagedKVCache: out of blocks")
            blocks = [self.free.pop() for _ in range(need - have)]
            if slot in self.tables:
                self.tables[slot].extend(blocks)
            else:
                self.tables[slot] = blocks
                self.seq_lens[slot] = 0

    def free_slot(self, slot: int) -> None:
        """free_slot (:77-89): zero the blocks, return them to the free list."""
        blocks = self.tables.pop(slot, [])
        for layer in range(self.num_layers):
            for b in blocks:
                self.k[layer][b].zero_()
                self.v[layer][b].zero_()
        self.free.extend(blocks)
        self.seq_lens.pop(slot, None)


def attention_with_kvcache(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                           k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: list[int],
                           cache_seqlen: int, scale: float) -> torch.Tensor:
    """flash_attn_with_kvcache semantics (worker_sync.py:196-203) for one slot.

    q [T, Hq, D], k_new/v_new [T, Hkv, D]: the new keys/values are written
    into the paged cache at positions cache_seqlen .. cache_seqlen+T-1, then
    query t attends causally to cache positions 0 .. cache_seqlen + t (GQA:
    query head h uses kv head h // (Hq / Hkv)). Returns [T, Hq, D] bf16.
    """
    T, Hq, D = q.shape
    Hkv = k_new.shape[1]
    bs = k_cache.shape[1]
    for t in range(T):
        pos = cache_seqlen + t
        blk = block_table[pos // bs]
        k_cache[blk, pos % bs] = k_new[t]
        v_cache[blk, pos % bs] = v_new[t]
    L = cache_seqlen + T
    idx = torch.arange(L)
    blocks = torch.tensor([block_table[p // bs] for p in range(L)], dtype=torch.long)
    K = k_cache[blocks, idx % bs].float()  # [L, Hkv, D]
    V = v_cache[blocks, idx % bs].float()
    group = Hq // Hkv
    K = K.repeat_interleave(group, 1)  # [L, Hq, D]
    V = V.repeat_interleave(group, 1)
    s = torch.einsum("thd,lhd->htl", q.float(), K) * scale
    mask = idx[None, :] > (cache_seqlen + torch.arange(T))[:, None]  # [T, L]
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, -1)
    o = torch.einsum("htl,lhd->thd", p, V)
    return bf(o)
