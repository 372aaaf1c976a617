"""Donor weight transfer on the CPU: the dict export_weight_ipc_handles builds
has the reference's keys (ext_aggregator.cpp:1216-1291) plus the offsets,
import_weights_from_ipc turns such a dict (or a reference dict without
offsets) back into the same records, and the library rejects malformed
exports before it touches a GPU."""
import ctypes as C

import pytest

from swarmlora_b200 import _native
from swarmlora_b200 import ext_aggregator as agg

L = 2
DIMS = [(512, 256, 256, 1024, 1024), (512, 256, 256, 1024, 1024)]


def _records():
    """(handle, offset, rows, cols) per record: layer 0 has an o bias."""
    out = []
    for l, (q, k, v, g, u) in enumerate(DIMS):
        out += [(bytes([l + 1]) * 64, 0, q + k + v, 512), (bytes([9]) * 64, 1024 + l, 512, 512),
                (bytes([l + 3]) * 64, 0, g + u, 512), (bytes([9]) * 64, 4096 + l, 512, 1024),
                ((bytes([9]) * 64, 8192, 512, 1) if l == 0 else (bytes(64), 0, 0, 0)), (bytes(64), 0, 0, 0)]
    out += [(bytes([9]) * 64, 1 << 20, 2048, 512), (bytes([9]) * 64, 1 << 21, 2048, 512)]
    return out


class FakeLib:
    def __init__(self):
        self.imported = None

    def swl_agg_export_weights(self, recs, cap, dims, nl, dev):
        C.cast(nl, C.POINTER(C.c_int))[0] = L
        C.cast(dev, C.POINTER(C.c_int))[0] = 3
        if not recs:
            return 0
        for i, (h, off, rows, cols) in enumerate(_records()):
            C.memmove(recs[i].handle, h, 64)
            recs[i].offset, recs[i].rows, recs[i].cols = off, rows, cols
        for l, d in enumerate(DIMS):
            for j, x in enumerate(d):
                dims[5 * l + j] = x
        return 0

    def swl_agg_import_weights(self, recs, n, dims, nl, dev):
        self.imported = ([(bytes(recs[i].handle), recs[i].offset, recs[i].rows, recs[i].cols) for i in range(n)],
                         [dims[i] for i in range(5 * nl)], nl, dev)
        return 0


@pytest.fixture
def fake(monkeypatch):
    f = FakeLib()
    monkeypatch.setattr(agg, "lib", lambda: f)
    return f


def test_export_dict_has_the_reference_keys(fake):
    d = agg.export_weight_ipc_handles()
    assert d["num_layers"] == L and d["device_index"] == 3 and d["dtype_code"] == 15
    l0, l1 = d["layers"]
    for name in ("qkv_weight", "o_weight", "gate_up_weight", "down_weight"):
        assert len(l0[f"{name}_handle"]) == 64 and len(l0[f"{name}_shape"]) == 2
    assert l0["qkv_weight_shape"] == (1024, 512) and l0["down_weight_shape"] == (512, 1024)
    assert l0["o_weight_offset"] == 1024 and l1["down_weight_offset"] == 4097
    assert l0["has_o_bias"] and l0["o_bias_size"] == 512 and l0["o_bias_offset"] == 8192
    assert not l0["has_down_bias"] and not l1["has_o_bias"] and "o_bias_handle" not in l1
    assert [l0[k] for k in ("q_dim", "k_dim", "v_dim", "gate_dim", "up_dim")] == list(DIMS[0])
    assert d["embed_weight_shape"] == (2048, 512) and d["lm_head_weight_offset"] == 1 << 21


def test_import_turns_the_dict_back_into_records(fake):
    d = agg.export_weight_ipc_handles()
    agg.import_weights_from_ipc(d, 5)
    recs, dims, nl, dev = fake.imported
    assert recs == _records() and dims == [x for dd in DIMS for x in dd] and (nl, dev) == (L, 5)
    # a dict from the reference's own export has no offsets: weights at offset 0
    ref = {k: v for k, v in d.items() if not k.endswith("_offset")}
    ref["layers"] = [{k: v for k, v in lh.items() if not k.endswith("_offset")} for lh in d["layers"]]
    agg.import_weights_from_ipc(ref, 0)
    assert all(r[1] == 0 for r in fake.imported[0])


def test_import_rejects_malformed_dicts(fake):
    d = agg.export_weight_ipc_handles()
    with pytest.raises(RuntimeError, match="bf16"):
        agg.import_weights_from_ipc(dict(d, dtype_code=6), 0)
    with pytest.raises(RuntimeError, match="layer entries"):
        agg.import_weights_from_ipc(dict(d, num_layers=3), 0)
    bad = dict(d, layers=[dict(d["layers"][0], qkv_weight_handle=b"x" * 10), d["layers"][1]])
    with pytest.raises(RuntimeError, match="64 bytes"):
        agg.import_weights_from_ipc(bad, 0)


def test_library_checks_records_before_any_cuda_call():
    """The real library: shape disagreements are refused before mapping."""
    lib = _native.lib()
    n = 6 * L + 2
    recs = (_native.WeightIpc * n)()
    for i, (h, off, rows, cols) in enumerate(_records()):
        C.memmove(recs[i].handle, h, 64)
        recs[i].offset, recs[i].rows, recs[i].cols = off, rows, cols
    dims = (C.c_int64 * (5 * L))(*[x for dd in DIMS for x in dd])
    assert lib.swl_agg_import_weights(recs, n - 1, dims, L, 0) != 0
    assert "records" in _native.last_error()
    recs[0].rows += 1  # qkv rows != q + k + v
    assert lib.swl_agg_import_weights(recs, n, dims, L, 0) != 0
    assert "layer 0 shapes disagree" in _native.last_error()
    recs[0].rows -= 1
    recs[6 * L + 1].cols = 256  # lm_head hidden != embed hidden
    assert lib.swl_agg_import_weights(recs, n, dims, L, 0) != 0
    assert "embed / lm_head" in _native.last_error()
    recs[6 * L + 1].cols = 512
    dims[3] = 0
    assert lib.swl_agg_import_weights(recs, n, dims, L, 0) != 0
    assert "dimension" in _native.last_error()
    assert lib.swl_agg_export_weights(None, 0, None, None, None) != 0
    assert "not initialized" in _native.last_error()
