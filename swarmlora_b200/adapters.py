"""LoRA adapter directories in the PEFT layout the reference's workers load
(adapter_config.json + adapter_model.safetensors), read into the per-layer
form `SlotGroup.pack_adapter` takes.

Follows the reference's loader, src/worker/model_builder.py:
  * `_validate_adapter_id` (:63-89): ids with NUL, empty or longer than 512
    characters are refused; a local path must resolve under one of the
    allowed base directories, or, with none registered, may not use `..`;
  * `_load_lora_raw` (:113-134): the config's `r` and `lora_alpha` (default
    r), every tensor of adapter_model.safetensors cast to bf16, a `.bin`
    file refused (pickle), no weights a FileNotFoundError;
  * `load_lora_fast` (:137-183): keys
    `base_model.model.model.layers.{i}.{self_attn|mlp}.{proj}.lora_{A|B}.weight`,
    scaling = lora_alpha / r (rsLoRA and per-module rank patterns are not
    applied there either).
A projection the file leaves out gets zero A and B, as FusedLoRA packs a
missing member (model_builder.py:228-233), so its delta is exactly zero.
Hub ids are not resolved (no download on the data path).

The file is read into one pinned host staging buffer that the loader keeps
and reuses, and reaches the GPU as one host-to-device copy; the tensors are
views into that device copy, cast to bf16 there.
"""
from __future__ import annotations

import json
import os
import re
import struct

import torch

MODULES = {"q": "self_attn", "k": "self_attn", "v": "self_attn", "o": "self_attn",
           "gate": "mlp", "up": "mlp", "down": "mlp"}
_KEY = re.compile(r"^base_model\.model\.model\.layers\.(\d+)\.(self_attn|mlp)\.([a-z]+)_proj\.lora_(A|B)\.weight$")
_DTYPES = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16}


def module_dims(cfg) -> dict:
    """(in_features, out_features) of each LoRA target for a model config."""
    H, I, D = cfg.hidden, cfg.inter, cfg.head_dim
    return {"q": (H, cfg.hq * D), "k": (H, cfg.hkv * D), "v": (H, cfg.hkv * D), "o": (cfg.hq * D, H),
            "gate": (H, I), "up": (H, I), "down": (I, H)}


def validate_adapter_id(path: str, allowed_bases=()) -> str:
    """The resolved directory of a local adapter id, or ValueError /
    FileNotFoundError as the reference's checks give."""
    if not path or "\x00" in path or len(path) > 512:
        raise ValueError(f"Invalid adapter ID: {path!r}")
    real = os.path.realpath(path)
    bases = [os.path.realpath(b) for b in allowed_bases]
    if bases:
        if not any(real == b or real.startswith(b + os.sep) for b in bases):
            raise ValueError(f"Adapter path outside allowed directories: {path!r}")
    elif ".." + os.sep in path or path.endswith(".."):
        raise ValueError(f"Path traversal rejected: {path!r}")
    if not os.path.isdir(real):
        raise FileNotFoundError(f"No adapter directory at {path!r}")
    return real


def _parse_header(f, size: int):
    """safetensors layout: little-endian u64 header length, JSON header of
    {name: {dtype, shape, data_offsets: [begin, end]}} (offsets from the
    end of the header), then the data."""
    head = f.read(8)
    if len(head) != 8:
        raise ValueError("adapter_model.safetensors: truncated header")
    n = struct.unpack("<Q", head)[0]
    if n > size - 8:
        raise ValueError("adapter_model.safetensors: header longer than the file")
    header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    return header, 8 + n


class AdapterLoader:
    """Reads adapter directories for one model config onto one device.
    Keeps a pinned staging buffer (grown on demand) and reuses it once the
    previous copy out of it has completed."""

    def __init__(self, cfg, device, allowed_bases=()):
        self.cfg = cfg
        self.device = torch.device(device)
        self.allowed_bases = tuple(allowed_bases)
        self._stage = None
        self._done = None  # event after the last copy out of the staging buffer

    def _staging(self, nbytes: int) -> torch.Tensor:
        if self._done is not None:
            self._done.synchronize()
        if self._stage is None or self._stage.numel() < nbytes:
            pin = self.device.type == "cuda"
            self._stage = torch.empty(nbytes, dtype=torch.uint8, pin_memory=pin)
        return self._stage[:nbytes]

    def load(self, path: str):
        """(layers, config): layers[l][proj] = (lora_A [r, in], lora_B [out, r])
        in bf16 on the device for every proj in MODULES; config is the
        adapter_config.json dict with `r`, `lora_alpha` and `scaling` set."""
        real = validate_adapter_id(path, self.allowed_bases)
        with open(os.path.join(real, "adapter_config.json")) as f:
            config = json.load(f)
        st = os.path.join(real, "adapter_model.safetensors")
        if not os.path.exists(st):
            if os.path.exists(os.path.join(real, "adapter_model.bin")):
                raise ValueError(f"Adapter at {path!r} uses .bin format which is not allowed. "
                                 f"Convert to safetensors format.")
            raise FileNotFoundError(f"No adapter weights found in {path!r}")
        r = int(config["r"])
        alpha = float(config.get("lora_alpha", r))
        if r < 1:
            raise ValueError(f"adapter {path!r}: rank {r}")
        size = os.path.getsize(st)
        with open(st, "rb") as f:
            header, data0 = _parse_header(f, size)
            stage = self._staging(size - data0)
            if f.readinto(memoryview(stage.numpy())) != stage.numel():
                raise ValueError("adapter_model.safetensors: truncated data")
        if self.device.type == "cuda":
            buf = stage.to(self.device, non_blocking=True)
            self._done = torch.cuda.Event()
            self._done.record(torch.cuda.current_stream(self.device))
        else:
            buf = stage.clone()
        dims = module_dims(self.cfg)
        found = {}
        for key, meta in header.items():
            m = _KEY.match(key)
            if m is None or m.group(3) not in MODULES or MODULES[m.group(3)] != m.group(2):
                raise ValueError(f"adapter {path!r}: unexpected tensor {key!r}")
            layer, proj, ab = int(m.group(1)), m.group(3), m.group(4)
            if layer >= self.cfg.layers:
                raise ValueError(f"adapter {path!r}: layer {layer} beyond the model's {self.cfg.layers}")
            dt = _DTYPES.get(meta["dtype"])
            if dt is None:
                raise ValueError(f"adapter {path!r}: {key} has dtype {meta['dtype']}")
            shape = tuple(int(s) for s in meta["shape"])
            k_in, n_out = dims[proj]
            want = (r, k_in) if ab == "A" else (n_out, r)
            if shape != want:
                raise ValueError(f"adapter {path!r}: {key} has shape {list(shape)}, expected {list(want)}")
            b, e = (int(x) for x in meta["data_offsets"])
            es = torch.tensor([], dtype=dt).element_size()
            if e - b != shape[0] * shape[1] * es or e > buf.numel():
                raise ValueError(f"adapter {path!r}: {key} has inconsistent data offsets")
            raw = buf[b:e] if b % es == 0 else buf[b:e].clone()
            found[(layer, proj, ab)] = raw.view(dt).view(shape).to(torch.bfloat16)
        layers = []
        for layer in range(self.cfg.layers):
            d = {}
            for proj, (k_in, n_out) in dims.items():
                A, B = found.get((layer, proj, "A")), found.get((layer, proj, "B"))
                if (A is None) != (B is None):
                    raise ValueError(f"adapter {path!r}: layer {layer} {proj}_proj has only one of lora_A / lora_B")
                if A is None:
                    A = torch.zeros(r, k_in, dtype=torch.bfloat16, device=self.device)
                    B = torch.zeros(n_out, r, dtype=torch.bfloat16, device=self.device)
                d[proj] = (A, B)
            layers.append(d)
        config = dict(config, r=r, lora_alpha=alpha, scaling=alpha / r)
        return layers, config


def load_adapter(path: str, cfg, device, allowed_bases=()):
    """One-off AdapterLoader(cfg, device, allowed_bases).load(path)."""
    return AdapterLoader(cfg, device, allowed_bases).load(path)


def save_adapter(path: str, layers: list, alpha: float, dtype=torch.float32, base_model: str = "") -> None:
    """Writes per-layer {proj: (lora_A, lora_B)} as a PEFT adapter directory
    (the layout the reference's adapter generator writes: fp32 tensors,
    every projection of every layer targeted)."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    r = int(layers[0]["q"][0].shape[0])
    tensors = {}
    for l, d in enumerate(layers):
        for proj, (A, B) in d.items():
            pre = f"base_model.model.model.layers.{l}.{MODULES[proj]}.{proj}_proj"
            tensors[f"{pre}.lora_A.weight"] = A.detach().to("cpu", dtype).contiguous()
            tensors[f"{pre}.lora_B.weight"] = B.detach().to("cpu", dtype).contiguous()
    save_file(tensors, os.path.join(path, "adapter_model.safetensors"))
    targets = sorted({f"{p}_proj" for d in layers for p in d})
    config = {"peft_type": "LORA", "task_type": "CAUSAL_LM", "base_model_name_or_path": base_model,
              "r": r, "lora_alpha": alpha, "lora_dropout": 0, "bias": "none", "fan_in_fan_out": False,
              "inference_mode": True, "target_modules": targets, "use_dora": False, "use_rslora": False}
    with open(os.path.join(path, "adapter_config.json"), "w") as f:
        json.dump(config, f, indent=2)
