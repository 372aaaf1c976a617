"""Direct access to the slot-round kernel over caller-owned buffers.

`slot_gemm` runs one gather -> GEMM -> scatter round over a list of per-slot
input tensors and writes each slot's output tensor in place: the operation
of the reference's execute_batched_gemm_slots (ext_aggregator.cpp:470-626)
without the slot pool around it. Used by tests and the benchmark; the
aggregator module runs the same kernel over its pool.
"""
from __future__ import annotations

import torch

from ._native import check, i32_array, lib, ptr_array

ALGO_AUTO, ALGO_TENSOR_CORE, ALGO_SIMT, ALGO_STREAM_K = 0, 1, 2, 3


def slot_gemm(W: torch.Tensor, inputs: list[torch.Tensor], outputs: list[torch.Tensor],
              bias: torch.Tensor | None = None, algo: int = ALGO_AUTO, splits: int = 0,
              stream: torch.cuda.Stream | None = None) -> None:
    """outputs[i][:rows_i] = inputs[i] @ W^T (+ bias) for every slot i.

    W: [N, K] bf16 CUDA, row-major. inputs[i]: [rows_i, K] bf16 with unit
    stride in K; outputs[i]: [>= rows_i, N] bf16 with unit stride in N. All
    slots must share the row strides of inputs[0] / outputs[0].
    """
    if W.dtype != torch.bfloat16 or not W.is_cuda or not W.is_contiguous():
        raise RuntimeError("slot_gemm: W must be a contiguous bf16 CUDA tensor")
    N, K = W.shape
    n = len(inputs)
    if n != len(outputs):
        raise RuntimeError("slot_gemm: inputs and outputs differ in length")
    rows = [int(x.shape[0]) for x in inputs]
    in_stride = int(inputs[0].stride(0)) if n else K
    out_stride = int(outputs[0].stride(0)) if n else N
    for x, y, r in zip(inputs, outputs, rows):
        if x.dtype != torch.bfloat16 or y.dtype != torch.bfloat16:
            raise RuntimeError("slot_gemm: slot buffers must be bf16")
        if x.shape[-1] != K or y.shape[-1] != N or y.shape[0] < r:
            raise RuntimeError("slot_gemm: slot buffer shape mismatch")
        if (r > 1 and (x.stride(0) != in_stride or y.stride(0) != out_stride)) or \
                x.stride(-1) != 1 or y.stride(-1) != 1:
            raise RuntimeError("slot_gemm: slot buffers must share row strides")
    st = stream if stream is not None else torch.cuda.current_stream(W.device)
    check(lib().swl_slot_gemm(
        W.data_ptr(), N, K, bias.data_ptr() if bias is not None else None, n,
        ptr_array([x.data_ptr() for x in inputs]), ptr_array([y.data_ptr() for y in outputs]),
        i32_array(rows), in_stride, out_stride, algo, splits, st.cuda_stream))


def device_error() -> int:
    """Synchronously reads and clears the round kernels' bounded-wait error word."""
    import ctypes
    code = ctypes.c_uint(0)
    check(lib().swl_round_device_error(ctypes.byref(code)))
    return int(code.value)


def next_tokens(logits: torch.Tensor, params, u: torch.Tensor | None = None, seed: int = 0, offset: int = 0,
                out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """The LM head's next token per row of bf16 logits [rows, >= vocab]
    (vocab = logits.shape[1] unless the rows are padded: pass a view).
    params: one (do_sample, temperature, top_k, top_p) per row; greedy rows
    take the argmax, sampling rows draw with the reference's temperature /
    top-k / top-p rule at u[row] (a float32 CUDA tensor) or at uniforms
    derived from (seed, offset, row). Returns int64 tokens on the device."""
    from ._native import Sampling
    if logits.dtype != torch.bfloat16 or not logits.is_cuda or logits.stride(-1) != 1:
        raise RuntimeError("next_tokens: logits must be bf16 CUDA with unit stride in the vocabulary")
    rows, vocab = int(logits.shape[0]), int(logits.shape[1])
    if len(params) != rows:
        raise RuntimeError("next_tokens: one parameter set per row")
    arr = (Sampling * max(1, rows))()
    for i, (d, t, k, p) in enumerate(params):
        arr[i].do_sample, arr[i].temperature, arr[i].top_k, arr[i].top_p = int(bool(d)), float(t), int(k), float(p)
    if u is not None and (u.dtype != torch.float32 or not u.is_cuda or u.numel() < rows):
        raise RuntimeError("next_tokens: u must be a float32 CUDA tensor with one value per row")
    out = out if out is not None else torch.empty(rows, dtype=torch.int64, device=logits.device)
    st = stream if stream is not None else torch.cuda.current_stream(logits.device)
    check(lib().swl_sample_rows(logits.data_ptr(), rows, vocab, int(logits.stride(0)), arr,
                                u.data_ptr() if u is not None else None, int(seed), int(offset), out.data_ptr(),
                                st.cuda_stream))
    return out
