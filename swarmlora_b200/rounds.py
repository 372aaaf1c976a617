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
