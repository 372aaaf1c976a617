"""Base-model checkpoints in the Hugging Face Llama layout the reference's
aggregator loads (AutoModelForCausalLM.from_pretrained, src/aggregator.py:
170-189, then init_aggregator_layer per layer, :330-356): config.json plus
model.safetensors or a sharded model.safetensors.index.json.

`load_base` reads the tensors the aggregator and the workers use
(q/k/v/o, gate/up/down, the two RMSNorm weights per layer, the final norm,
the embedding and the LM head — the embedding again when the weights are
tied) into a BaseWeights of bf16 tensors on one device, through a pinned
host staging buffer and one host-to-device copy per tensor. `config_from_hf`
maps config.json onto ModelConfig the way the reference reads it (head_dim
from hidden / heads when absent, rms_norm_eps 1e-6 when absent, :182-189).
"""
from __future__ import annotations

import json
import os

import torch

from .adapters import _DTYPES, _parse_header
from .engine import BaseWeights, ModelConfig

_LAYER = "model.layers.{}."
_PER_LAYER = {"q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
              "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
              "down": "mlp.down_proj.weight", "in_norm": "input_layernorm.weight",
              "post_norm": "post_attention_layernorm.weight"}


def config_from_hf(hf: dict, **overrides) -> ModelConfig:
    """ModelConfig of an HF Llama config.json (dict); overrides set the
    serving fields (rank, alpha, page, max_seq_per_step)."""
    H, hq = int(hf["hidden_size"]), int(hf["num_attention_heads"])
    # transformers 4 writes rope_theta + rope_scaling; 5 writes both in rope_parameters
    rp = dict(hf.get("rope_parameters") or {})
    theta = float(hf.get("rope_theta", rp.pop("rope_theta", 10000.0)))
    scaling = hf.get("rope_scaling") or (rp if rp.get("rope_type", "default") != "default" else None)
    fields = dict(hidden=H, inter=int(hf["intermediate_size"]), layers=int(hf["num_hidden_layers"]), hq=hq,
                  hkv=int(hf.get("num_key_value_heads") or hq), head_dim=int(hf.get("head_dim") or H // hq),
                  vocab=int(hf["vocab_size"]), eps=float(hf.get("rms_norm_eps", 1e-6)), rope_theta=theta,
                  rope_scaling=dict(scaling) if scaling else {})
    fields.update(overrides)
    return ModelConfig(**fields)


def _shards(path: str) -> dict:
    """{tensor name: shard file} of a checkpoint directory."""
    index = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            wm = json.load(f)["weight_map"]
        return {k: os.path.join(path, v) for k, v in wm.items()}
    single = os.path.join(path, "model.safetensors")
    if os.path.exists(single):
        return {None: single}
    if any(n.endswith(".bin") for n in os.listdir(path)):
        raise ValueError(f"checkpoint at {path!r} is pickled (.bin); convert it to safetensors")
    raise FileNotFoundError(f"no model.safetensors(.index.json) in {path!r}")


def load_base(path: str, device, cfg: ModelConfig | None = None) -> tuple[BaseWeights, ModelConfig]:
    """(BaseWeights, ModelConfig) of an HF Llama checkpoint directory, every
    tensor bf16 on `device`."""
    with open(os.path.join(path, "config.json")) as f:
        hf = json.load(f)
    cfg = cfg or config_from_hf(hf)
    dev = torch.device(device)
    names = {"model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"}
    for l in range(cfg.layers):
        names |= {_LAYER.format(l) + v for v in _PER_LAYER.values()}
    where = _shards(path)
    files: dict = {}
    for n in names:
        f = where.get(n, where.get(None))
        if f is not None:
            files.setdefault(f, []).append(n)
    tensors = {}
    stage, done = None, None
    for fname, wanted in files.items():
        size = os.path.getsize(fname)
        with open(fname, "rb") as fh:
            header, data0 = _parse_header(fh, size)
            for n in sorted(wanted, key=lambda k: header[k]["data_offsets"][0] if k in header else 0):
                if n not in header:
                    continue
                meta = header[n]
                dt = _DTYPES.get(meta["dtype"])
                if dt is None:
                    raise ValueError(f"{fname}: {n} has dtype {meta['dtype']}")
                b, e = (int(x) for x in meta["data_offsets"])
                shape = tuple(int(s) for s in meta["shape"])
                nbytes = e - b
                if nbytes != torch.tensor([], dtype=dt).element_size() * int(torch.Size(shape).numel()):
                    raise ValueError(f"{fname}: {n} has inconsistent data offsets")
                if done is not None:
                    done.synchronize()  # the previous copy out of the staging buffer has finished
                if stage is None or stage.numel() < nbytes:
                    stage = torch.empty(nbytes, dtype=torch.uint8, pin_memory=dev.type == "cuda")
                buf = stage[:nbytes]
                fh.seek(data0 + b)
                if fh.readinto(memoryview(buf.numpy())) != nbytes:
                    raise ValueError(f"{fname}: {n} is truncated")
                if dev.type == "cuda":
                    t = buf.to(dev, non_blocking=True)
                    done = torch.cuda.Event()
                    done.record(torch.cuda.current_stream(dev))
                else:
                    t = buf.clone()
                tensors[n] = t.view(dt).view(shape).to(torch.bfloat16)
    if "lm_head.weight" not in tensors:
        if not hf.get("tie_word_embeddings", False):
            raise ValueError(f"checkpoint at {path!r} has no lm_head.weight and untied embeddings")
        tensors["lm_head.weight"] = tensors.get("model.embed_tokens.weight")
    missing = sorted(n for n in names if n not in tensors)
    if missing:
        raise ValueError(f"checkpoint at {path!r} lacks {missing[:4]}{' ...' if len(missing) > 4 else ''}")
    H, I, D = cfg.hidden, cfg.inter, cfg.head_dim
    want = {"q": (cfg.hq * D, H), "k": (cfg.hkv * D, H), "v": (cfg.hkv * D, H), "o": (H, cfg.hq * D),
            "gate": (I, H), "up": (I, H), "down": (H, I), "in_norm": (H,), "post_norm": (H,)}
    per = {k: [] for k in _PER_LAYER}
    for l in range(cfg.layers):
        for k, suffix in _PER_LAYER.items():
            t = tensors[_LAYER.format(l) + suffix]
            if tuple(t.shape) != want[k]:
                raise ValueError(f"layer {l} {k}: shape {tuple(t.shape)}, the config says {want[k]}")
            per[k].append(t)
    for n, shape in (("model.embed_tokens.weight", (cfg.vocab, H)), ("lm_head.weight", (cfg.vocab, H)),
                     ("model.norm.weight", (H,))):
        if tuple(tensors[n].shape) != shape:
            raise ValueError(f"{n}: shape {tuple(tensors[n].shape)}, the config says {shape}")
    base = BaseWeights(q=per["q"], k=per["k"], v=per["v"], o=per["o"], gate=per["gate"], up=per["up"],
                       down=per["down"], in_norm=per["in_norm"], post_norm=per["post_norm"],
                       final_norm=tensors["model.norm.weight"], embed=tensors["model.embed_tokens.weight"],
                       lm_head=tensors["lm_head.weight"])
    return base, cfg
