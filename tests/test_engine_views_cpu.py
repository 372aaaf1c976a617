"""SlotGroup.subset on the CPU: the view's per-slot tables hold exactly the
active slots' entries, in group order, for every table a step passes to the
kernels (slot ids, worker ids, buffers, pages, positions, caches, the eight
LoRA tables of every layer), and a step's position advance covers the whole
group with zeros outside the view. The group's tables are fake addresses,
so nothing touches a GPU."""
import pytest

from swarmlora_b200 import engine
from swarmlora_b200._native import ptr_array

N, LAYERS = 5, 2
LORA = ("A_qkv", "B_qkv", "A_o", "B_o", "A_gu", "B_gu", "A_dn", "B_dn")


class _Ptr:
    def __init__(self, p):
        self.p = p

    def data_ptr(self):
        return self.p


def _fake_group():
    g = object.__new__(engine.SlotGroup)
    g.cfg = engine.ModelConfig(layers=LAYERS, vocab=128)
    g.fused, g.n = True, N
    g.slot_ids = [10 + i for i in range(N)]
    g.worker_ids = [1000 + i for i in range(N)]
    for j, name in enumerate(("a_in", "a_out", "a_h", "a_qkv", "a_tok", "a_bt", "a_sl")):
        setattr(g, name, ptr_array([(j + 1) << 20 | i << 8 for i in range(N)]))
    g.k_cache = [_Ptr(0x7000_0000 + l) for l in range(LAYERS)]
    g.v_cache = [_Ptr(0x8000_0000 + l) for l in range(LAYERS)]
    for j, name in enumerate(LORA):
        # slot 2 has no adapter (None entries), as a group built with one
        setattr(g, name, [ptr_array([None if i == 2 else (0x100 + j) << 24 | l << 16 | i for i in range(N)])
                          for l in range(LAYERS)])
    g._subset, g._slot_index, g._advance, g.graph = None, list(range(N)), {}, None
    return g


def test_view_tables_hold_the_active_slots():
    g = _fake_group()
    v = g.subset([4, 2, 1])
    act = [1, 2, 4]
    assert v.n == 3 and v._slot_index == act and v._subset == tuple(act) and v.graph is None
    assert list(v.a_sids) == [11, 12, 14] and list(v.a_wids) == [1001, 1002, 1004]
    assert list(v.a_rows) == [1, 1, 1] and list(v.a_ones) == [1, 1, 1]
    assert list(v.a_b8) == [8] * 3 and list(v.a_bH) == [2 * g.cfg.hidden] * 3
    for name in ("a_in", "a_out", "a_h", "a_qkv", "a_tok", "a_bt", "a_sl"):
        full = list(getattr(g, name))
        assert list(getattr(v, name)) == [full[i] for i in act], name
    for l in range(LAYERS):
        assert list(v.a_kc[l]) == [g.k_cache[l].p] * 3 and list(v.a_vc[l]) == [g.v_cache[l].p] * 3
        for name in LORA:
            full = list(getattr(g, name)[l])
            got = list(getattr(v, name)[l])
            assert got == [full[i] for i in act] and got[1] is None, (name, l)
    # the group itself is untouched
    assert g.n == N and g.slot_ids == [10, 11, 12, 13, 14] and g._subset is None
    assert len(list(g.a_in)) == N and len(list(g.A_qkv[0])) == N


def test_view_position_advance_covers_the_group():
    g = _fake_group()
    v = g.subset([0, 3])
    assert v._full_pattern(None) == [1, 0, 0, 1, 0]
    assert v._full_pattern([6, 1]) == [6, 0, 0, 1, 0]
    assert g._full_pattern([1, 2, 3, 4, 5]) == [1, 2, 3, 4, 5] and g._full_pattern(None) == [1] * N


def test_view_arguments_are_checked():
    g = _fake_group()
    with pytest.raises(ValueError):
        g.subset([])
    with pytest.raises(ValueError):
        g.subset([0, N])
    with pytest.raises(ValueError):
        g.subset([1]).subset([1])
    g.fused = False
    with pytest.raises(ValueError):
        g.subset([1])
