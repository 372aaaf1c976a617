"""CPU oracle for the SwarmLoRA aggregator hot path — TEST INFRASTRUCTURE ONLY.

A plain CPU restatement (torch on CPU, fp32 arithmetic rounded to bf16
wherever the reference materialises a bf16 tensor) of the reference's
per-token path: the gather -> base GEMM -> scatter round
(src/cpp_extensions/ext_aggregator.cpp:470-626), the worker's LoRA delta
(src/worker/model_builder.py:217-262, src/worker/worker_sync.py:305, :375),
NeoX RoPE + paged causal GQA attention (src/worker/worker_sync.py:168-205,
src/worker/paged_attention.py:7-142), the per-layer glue
(src/worker/worker_sync.py:1337-1425), embed and greedy LM head
(src/cpp_extensions/ext_aggregator.cpp:630-875).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package, and only as the checker / the timed CPU reference; the product
path (swarmlora_b200) never imports it.

Parity pinning: the LoRA packing and delta, the RoPE cos/sin cache and the
paged-KV block bookkeeping are pinned against golden vectors produced by
importing the reference's own Python modules (tests/golden/make_golden.py).
The reference has no test suite and no golden vectors of its own, and its
C++ round (cuBLAS via libtorch) cannot run on this CPU-only machine; the round
restatement (cat + x @ W^T in fp32, rounded to bf16 + per-slot split) is
pinned by construction and checked against HF transformers' LlamaDecoderLayer
for the whole layer (tests/test_oracle.py).
"""
