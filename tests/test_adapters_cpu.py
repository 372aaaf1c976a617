"""Adapter directories (swarmlora_b200.adapters) on the CPU, pinned against
the reference: the fixtures under tests/golden/adapter_* were written by the
reference's adapter generator, and adapter_load.pt holds what the reference's
loader (model_builder.py:137-183, load_lora_fast) read from them
(tests/golden/make_golden.py)."""
import json
import os
from pathlib import Path

import pytest
import torch

from swarmlora_b200 import adapters as ad
from swarmlora_b200 import worker_ops as wo
from swarmlora_b200.engine import ModelConfig

GOLDEN = Path(__file__).resolve().parent / "golden"
TINY = ModelConfig(hidden=64, inter=96, layers=2, hq=2, hkv=1, head_dim=32, vocab=128, rank=16, alpha=32)
MOD_NAME = {p: f"{ad.MODULES[p]}.{p}_proj" for p in ad.MODULES}


@pytest.fixture(scope="module")
def golden():
    return torch.load(GOLDEN / "adapter_load.pt", weights_only=False)


@pytest.mark.parametrize("name", ["adapter_r4", "adapter_r8_partial"])
def test_reader_matches_the_reference_loader(golden, name):
    want = golden[name]
    layers, config = ad.load_adapter(str(GOLDEN / name), TINY, "cpu")
    assert config["r"] == want["r"] and config["lora_alpha"] == want["lora_alpha"]
    assert config["scaling"] == want["lora_alpha"] / want["r"]
    assert len(layers) == TINY.layers
    for l, d in enumerate(layers):
        for proj, (A, B) in d.items():
            assert A.dtype == B.dtype == torch.bfloat16
            ref = want["modules"].get((l, MOD_NAME[proj]))
            if ref is None:  # a projection the file leaves out: exact zeros
                assert not A.any() and not B.any(), (name, l, proj)
                assert A.shape == (want["r"], ad.module_dims(TINY)[proj][0])
                continue
            rA, rB, rs = ref
            assert torch.equal(A, rA) and torch.equal(B, rB), (name, l, proj)
            assert rs == config["scaling"]
    if name == "adapter_r8_partial":
        assert not any((l, MOD_NAME["v"]) in want["modules"] for l in range(2))
        assert not layers[0]["v"][0].any() and not layers[1]["down"][1].any()


def test_packed_loaded_adapter_keeps_the_reference_prescale(golden):
    """QKV's A is A.t() * (lora_alpha / r) in bf16 (model_builder.py:237);
    the missing v block packs to zeros; padding to the group's rank adds
    zero columns."""
    layers, config = ad.load_adapter(str(GOLDEN / "adapter_r8_partial"), TINY, "cpu")
    s = config["scaling"]
    R = TINY.rank
    L = wo.pack_lora_layer(layers[1], s, pad_rank=R, post_scale=TINY.alpha / R)
    A_q, A_k, A_v = (L.A_qkv[:, i * R:(i + 1) * R] for i in range(3))
    rq = golden["adapter_r8_partial"]["modules"][(1, MOD_NAME["q"])][0]
    assert torch.equal(A_q[:, :8], rq.t() * s) and not A_q[:, 8:].any()
    assert not A_v.any()
    assert torch.equal(A_k[:, :8], golden["adapter_r8_partial"]["modules"][(1, MOD_NAME["k"])][0].t() * s)


def test_save_then_load_round_trip(scratch):
    g = torch.Generator().manual_seed(3)
    dims = ad.module_dims(TINY)
    layers = [{p: ((torch.randn(8, i, generator=g) * 0.05).to(torch.bfloat16),
                   (torch.randn(o, 8, generator=g) * 0.05).to(torch.bfloat16)) for p, (i, o) in dims.items()}
              for _ in range(TINY.layers)]
    ad.save_adapter(str(scratch / "a"), layers, alpha=16)
    loader = ad.AdapterLoader(TINY, "cpu")
    for _ in range(2):  # the staging buffer is reused
        got, config = loader.load(str(scratch / "a"))
        assert config["scaling"] == 2.0
        for l in range(TINY.layers):
            for p in dims:
                assert torch.equal(got[l][p][0], layers[l][p][0]) and torch.equal(got[l][p][1], layers[l][p][1])


def test_loader_refuses_what_the_reference_refuses(scratch):
    base = scratch / "pool"
    (base / "bin_only").mkdir(parents=True)
    (base / "bin_only" / "adapter_config.json").write_text(json.dumps({"r": 4}))
    (base / "bin_only" / "adapter_model.bin").write_bytes(b"\x80")
    with pytest.raises(ValueError, match=r"\.bin"):
        ad.load_adapter(str(base / "bin_only"), TINY, "cpu")
    (base / "empty").mkdir()
    (base / "empty" / "adapter_config.json").write_text(json.dumps({"r": 4}))
    with pytest.raises(FileNotFoundError):
        ad.load_adapter(str(base / "empty"), TINY, "cpu")
    with pytest.raises(ValueError, match="traversal"):
        ad.load_adapter(str(base / "empty") + "/../empty", TINY, "cpu")
    with pytest.raises(ValueError, match="Invalid"):
        ad.load_adapter("a\x00b", TINY, "cpu")
    with pytest.raises(ValueError, match="outside allowed"):
        ad.load_adapter(str(GOLDEN / "adapter_r4"), TINY, "cpu", allowed_bases=[str(base)])
    with pytest.raises(FileNotFoundError):
        ad.load_adapter(str(base / "nothing_here"), TINY, "cpu", allowed_bases=[str(base)])
    wide = ModelConfig(hidden=128, inter=96, layers=2, hq=2, hkv=1, head_dim=32, rank=16)
    with pytest.raises(ValueError, match="shape"):
        ad.load_adapter(str(GOLDEN / "adapter_r4"), wide, "cpu")
    one_layer = ModelConfig(hidden=64, inter=96, layers=1, hq=2, hkv=1, head_dim=32, rank=16)
    with pytest.raises(ValueError, match="beyond"):
        ad.load_adapter(str(GOLDEN / "adapter_r4"), one_layer, "cpu")
    from safetensors.torch import save_file
    (base / "extra").mkdir()
    (base / "extra" / "adapter_config.json").write_text(json.dumps({"r": 4}))
    save_file({"base_model.model.lm_head.lora_A.weight": torch.zeros(4, 64)},
              os.path.join(base / "extra", "adapter_model.safetensors"))
    with pytest.raises(ValueError, match="unexpected"):
        ad.load_adapter(str(base / "extra"), TINY, "cpu")
