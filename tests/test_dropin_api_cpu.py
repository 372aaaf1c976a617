"""The drop-in boundary seen from the reference's side: every call the
reference's Python makes on ext_aggregator, ext_ipc_queue and
ext_unified_barrier (tests/golden/reference_api_calls.json, read from
src/aggregator.py and src/worker/*.py by tests/golden/make_api_calls.py)
binds to this build's module of the same name — same function, the same
number of positional arguments, the same keyword names — and every module
attribute it reads exists with the reference's value."""
import inspect
import json
from pathlib import Path

import pytest

from swarmlora_b200 import ext_aggregator, ext_ipc_queue, ext_unified_barrier

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "reference_api_calls.json").read_text())
MODULES = {"ext_aggregator": ext_aggregator, "ext_ipc_queue": ext_ipc_queue,
           "ext_unified_barrier": ext_unified_barrier}
# op codes of the shared-memory protocol (ipc_types.h:19-25)
OP_CODES = {"OP_O_PROJ": 3, "OP_DOWN_PROJ": 6, "OP_QKV_FUSED": 9, "OP_GATE_UP_FUSED": 10, "OP_EMBED": 11,
            "OP_LM_HEAD": 12}


@pytest.mark.parametrize("call", GOLDEN["calls"], ids=lambda c: f"{c['module']}.{c['name']}")
def test_reference_call_binds(call):
    mod = MODULES[call["module"]]
    fn = getattr(mod, call["name"], None)
    assert callable(fn), f"{call['module']} has no {call['name']}"
    sig = inspect.signature(fn)
    sig.bind(*([None] * call["positional"]), **{k: None for k in call["keywords"]})


@pytest.mark.parametrize("attr", GOLDEN["attributes"], ids=lambda a: f"{a['module']}.{a['name']}")
def test_reference_attribute_exists(attr):
    mod = MODULES[attr["module"]]
    assert hasattr(mod, attr["name"]), f"{attr['module']} has no {attr['name']}"
    if attr["name"] in OP_CODES:
        assert getattr(mod, attr["name"]) == OP_CODES[attr["name"]]


def test_the_scan_saw_the_whole_protocol():
    names = {(c["module"], c["name"]) for c in GOLDEN["calls"]}
    for must in (("ext_aggregator", "aggregator_main_loop_slots"), ("ext_ipc_queue", "submit_slot_command"),
                 ("ext_ipc_queue", "wait_for_epoch"), ("ext_unified_barrier", "get_outputs_slot"),
                 ("ext_aggregator", "import_weights_from_ipc")):
        assert must in names
