"""Worker-side kernels (LoRA delta, RoPE + paged KV append, paged attention,
RMSNorm) over one or many slots, through libswarmlora_b200.so.

A worker process normally calls these for its single slot; the benchmark
calls them for all slots at once. Adapter weights are packed once into the
layouts the kernels read (`pack_lora_layer`), following the reference's
FusedLoRA packing (model_builder.py:217-262): the fused QKV / Gate+Up A
matrices are pre-scaled by alpha/r in bf16, O / Down scale after the expand
(worker_sync.py:305, :375).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from ._native import check, i32_array, lib, ptr_array

EXPAND_ADD, EXPAND_RESIDUAL, EXPAND_SILU_MUL = 0, 1, 2


def _stream(stream):
    return (stream if stream is not None else torch.cuda.current_stream()).cuda_stream


def _ptrs(ts):
    return ptr_array([t.data_ptr() if t is not None else None for t in ts])


@dataclass
class LoraLayer:
    """One layer of one adapter, in kernel layout (all bf16, on device)."""
    A_qkv: torch.Tensor   # [H, 3r]  = cat(Aq^T s, Ak^T s, Av^T s)
    B_qkv: torch.Tensor   # [q+k+v, r] = cat(Bq, Bk, Bv)
    A_o: torch.Tensor     # [H, r]   = Ao^T
    B_o: torch.Tensor     # [H, r]
    A_gu: torch.Tensor    # [H, 2r]  = cat(Ag^T s, Au^T s)
    B_gu: torch.Tensor    # [2I, r]  = cat(Bg, Bu)
    A_down: torch.Tensor  # [I, r]   = Ad^T
    B_down: torch.Tensor  # [H, r]
    rank: int
    scaling: float


def pack_lora_layer(w: dict, scaling: float, pad_rank: int | None = None,
                    post_scale: float | None = None) -> LoraLayer:
    """w maps 'q','k','v','o','gate','up','down' -> (lora_A [r, in], lora_B [out, r]).

    pad_rank packs the adapter at a larger rank (a group whose adapters have
    different ranks runs its kernels at the largest): A and B get zero
    columns, which add exact zeros, so the deltas are bit-identical.
    post_scale is the scale the O / Down kernels apply after the expand (one
    value per launch); the adapter's own `scaling` is reached by folding
    scaling / post_scale into its O and Down lora_B, which is exact when that
    ratio is a power of two (alpha / r for r in {8, 16, 32} and one alpha)."""
    r = int(w["q"][0].shape[0])
    R = int(pad_rank) if pad_rank else r
    if R < r:
        raise ValueError(f"pad_rank {R} below the adapter's rank {r}")
    fold = 1.0 if post_scale is None else float(scaling) / float(post_scale)

    def pad(t):  # [rows, r] -> [rows, R]
        return torch.nn.functional.pad(t, (0, R - t.shape[1])) if R > t.shape[1] else t

    def a_scaled(name):
        return pad((w[name][0].t() * scaling).to(torch.bfloat16))  # A.t() * s in bf16 (model_builder.py:237)

    def b_folded(name):
        b = w[name][1]
        return pad((b.float() * fold).to(torch.bfloat16) if fold != 1.0 else b)

    return LoraLayer(
        A_qkv=torch.cat([a_scaled("q"), a_scaled("k"), a_scaled("v")], 1).contiguous(),
        B_qkv=torch.cat([pad(w["q"][1]), pad(w["k"][1]), pad(w["v"][1])], 0).contiguous(),
        A_o=pad(w["o"][0].t()).contiguous(),
        B_o=b_folded("o").contiguous(),
        A_gu=torch.cat([a_scaled("gate"), a_scaled("up")], 1).contiguous(),
        B_gu=torch.cat([pad(w["gate"][1]), pad(w["up"][1])], 0).contiguous(),
        A_down=pad(w["down"][0].t()).contiguous(),
        B_down=b_folded("down").contiguous(),
        rank=R,
        scaling=float(post_scale) if post_scale is not None else float(scaling),
    )


LORA_FIELDS = ("A_qkv", "B_qkv", "A_o", "B_o", "A_gu", "B_gu", "A_down", "B_down")
_SLAB_ALIGN = 256  # elements: every tensor of a slab starts on a 512-byte boundary, as torch allocates


@dataclass
class PackedAdapter:
    """All layers of one adapter in one contiguous bf16 buffer (`slab`);
    `layers` are LoraLayers whose tensors are views into it. Adapters packed
    at the same rank for the same model share the layout, so a slot's adapter
    is replaced by one device copy of the slab."""
    slab: torch.Tensor
    layers: list
    rank: int            # the adapter's own rank (the slab holds it padded)


def pack_lora_slab(layers: list, rank: int | None = None) -> PackedAdapter:
    """Copies packed layers (pack_lora_layer) into one slab, fields in
    LORA_FIELDS order layer after layer."""
    offs, total = [], 0
    for L in layers:
        row = []
        for f in LORA_FIELDS:
            t = getattr(L, f)
            row.append((total, tuple(t.shape)))
            total += -(-t.numel() // _SLAB_ALIGN) * _SLAB_ALIGN
        offs.append(row)
    slab = torch.empty(total, dtype=torch.bfloat16, device=layers[0].A_qkv.device)
    views = []
    for L, row in zip(layers, offs):
        kw = {}
        for f, (o, shape) in zip(LORA_FIELDS, row):
            n = shape[0] * shape[1]
            v = slab[o:o + n].view(shape)
            v.copy_(getattr(L, f))
            kw[f] = v
        views.append(LoraLayer(**kw, rank=L.rank, scaling=L.scaling))
    return PackedAdapter(slab, views, int(rank) if rank is not None else layers[0].rank)


def lora_shrink(xs, As, K: int, R: int, splits: int, ws: torch.Tensor, x_stride: int | None = None,
                rows=None, stream=None) -> None:
    rows = rows if rows is not None else [int(x.shape[0]) for x in xs]
    x_stride = x_stride if x_stride is not None else int(xs[0].stride(0))
    check(lib().swl_lora_shrink(len(xs), i32_array(rows), _ptrs(xs), x_stride, _ptrs(As), K, R,
                                splits, ws.data_ptr(), _stream(stream)))


def lora_expand(bases, Bs, outs, n_total: int, r: int, block_ends, mode: int, splits: int,
                ws: torch.Tensor, resids=None, post_scale: float = 0.0, rows=None,
                base_stride: int | None = None, out_stride: int | None = None,
                resid_stride: int = 0, stream=None) -> None:
    rows = rows if rows is not None else [int(b.shape[0]) for b in bases]
    base_stride = base_stride if base_stride is not None else int(bases[0].stride(0))
    out_stride = out_stride if out_stride is not None else int(outs[0].stride(0))
    be = (C.c_int64 * 3)(*[int(x) for x in block_ends] + [n_total] * (3 - len(block_ends)))
    check(lib().swl_lora_expand(
        len(bases), i32_array(rows), _ptrs(bases), base_stride,
        _ptrs(Bs) if Bs is not None else None,
        _ptrs(resids) if resids is not None else None, resid_stride,
        _ptrs(outs), out_stride, n_total, r, len(block_ends), be, float(post_scale), mode, splits,
        ws.data_ptr(), _stream(stream)))


def rope_append(qkvs, block_tables, k_caches, v_caches, seqlens, q_rot, cos_sin, hq: int, hkv: int,
                head_dim: int = 128, page: int = 16, rows=None, qkv_stride: int | None = None,
                stream=None) -> None:
    rows = rows if rows is not None else [int(q.shape[0]) for q in qkvs]
    qkv_stride = qkv_stride if qkv_stride is not None else int(qkvs[0].stride(0))
    check(lib().swl_rope_append(len(qkvs), i32_array(rows), _ptrs(qkvs), qkv_stride,
                                _ptrs(block_tables), _ptrs(k_caches), _ptrs(v_caches),
                                _ptrs(seqlens), hq, hkv, head_dim, page, cos_sin.data_ptr(),
                                int(cos_sin.shape[0]), q_rot.data_ptr(), _stream(stream)))


def attention_tune(chunk_pages: int = 0, stages: int = 0, groups: int = 0) -> None:
    """Pages per context chunk, page-ring depth and kv head groups (CTAs that
    share one page's heads) of the attention launch (0 = automatic)."""
    check(lib().swl_attention_tune(chunk_pages, stages, groups))


def attention_tma(on: bool = True) -> None:
    """K/V pages by TMA (default, when every row's pages share one cache
    allocation) or by per-lane copies."""
    check(lib().swl_attention_tma(1 if on else 0))


def attention_part_floats(total_rows: int, hq: int, hkv: int, max_len: int) -> int:
    return int(lib().swl_attention_part_floats(total_rows, hq, hkv, max_len))


def paged_attention(rows, block_tables, k_caches, v_caches, seqlens, outs, q_rot, part, hq: int,
                    hkv: int, max_len: int, scale: float, head_dim: int = 128, page: int = 16,
                    out_stride: int | None = None, stream=None) -> None:
    out_stride = out_stride if out_stride is not None else int(outs[0].stride(0))
    check(lib().swl_paged_attention(len(rows), i32_array(rows), _ptrs(block_tables),
                                    _ptrs(k_caches), _ptrs(v_caches), _ptrs(seqlens), _ptrs(outs),
                                    out_stride, hq, hkv, head_dim, page, float(scale), max_len,
                                    q_rot.data_ptr(), part.data_ptr() if part is not None else None,
                                    _stream(stream)))


def paged_attention_noalloc(rows, block_tables, k_caches, v_caches, seqlens, outs, q_rot, hq: int,
                            hkv: int, max_len: int, scale: float, head_dim: int = 128,
                            page: int = 16, out_stride: int | None = None, stream=None) -> None:
    """paged_attention with its partials in the library's static per-device
    array (NOALLOC_ATTN_SCRATCH_FLOATS fp32): allocates nothing. Calls that
    overlap on the GPU share that array and must not run concurrently."""
    out_stride = out_stride if out_stride is not None else int(outs[0].stride(0))
    check(lib().swl_paged_attention_noalloc(len(rows), i32_array(rows), _ptrs(block_tables),
                                            _ptrs(k_caches), _ptrs(v_caches), _ptrs(seqlens),
                                            _ptrs(outs), out_stride, hq, hkv, head_dim, page,
                                            float(scale), max_len, q_rot.data_ptr(),
                                            _stream(stream)))


NOALLOC_ATTN_SCRATCH_FLOATS = 1 << 20


def rms_norm(xs, outs, w: torch.Tensor, eps: float, rows=None, x_stride: int | None = None,
             out_stride: int | None = None, stream=None) -> None:
    rows = rows if rows is not None else [int(x.shape[0]) for x in xs]
    x_stride = x_stride if x_stride is not None else int(xs[0].stride(0))
    out_stride = out_stride if out_stride is not None else int(outs[0].stride(0))
    check(lib().swl_rms_norm(len(xs), i32_array(rows), _ptrs(xs), x_stride, _ptrs(outs),
                             out_stride, w.data_ptr(), int(w.shape[0]), float(eps),
                             _stream(stream)))
