"""C-ABI boundary checks that need no GPU: the library loads, the public header
compiles as plain C, and the header's declarations and the library's exports
are the same set of symbols (and match the Python binding's table)."""
import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "swarmlora_b200.h"


def _header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(swl_[a-z0-9_]+)\s*\(", text))


def _exported(native):
    out = subprocess.run(["nm", "-D", "--defined-only", str(native.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T swl_" in line}


def test_library_loads(native):
    lib = native.lib()
    assert lib.swl_abi_version() == 1
    assert native.last_error() is not None


def test_header_matches_exports(native):
    declared = _header_functions()
    exported = _exported(native)
    assert declared == exported, (
        f"declared only: {sorted(declared - exported)}; exported only: {sorted(exported - declared)}")


def test_python_binding_covers_exports(native):
    exported = _exported(native)
    bound = set(native.SIGNATURES)
    assert exported <= bound, f"unbound exports: {sorted(exported - bound)}"


def test_header_compiles_as_c(scratch):
    src = scratch / "use.c"
    src.write_text('#include "swarmlora_b200.h"\nint main(void){return swl_abi_version() == 1 ? 0 : 1;}\n')
    res = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", f"-I{ROOT / 'include'}",
                          str(src)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


def test_errors_are_reported_without_gpu(native):
    """Calls that fail before touching the device return a status and a message."""
    lib = native.lib()
    assert lib.swl_q_init_batch_control(4) != 0
    assert "not initialized" in native.last_error()
    assert lib.swl_agg_claim_slot(1, None, None, None, None, None) != 0
    assert "not initialized" in native.last_error()
    assert lib.swl_agg_get_slot_owner(0) == -1


def test_sampling_entry_points_check_arguments(native):
    """swl_sample_rows and swl_agg_set_worker_sampling refuse bad arguments
    with a message, before any device work."""
    import ctypes as C
    lib = native.lib()
    p = (native.Sampling * 2)()
    out = C.c_void_p(0x1000)
    assert lib.swl_sample_rows(C.c_void_p(0x1000), 200, 10, 10, p, None, 0, 0, out, None) != 0  # too many rows
    assert "sample" in native.last_error()
    assert lib.swl_sample_rows(C.c_void_p(0x1000), 2, 10, 5, p, None, 0, 0, out, None) != 0  # ld < vocab
    assert lib.swl_sample_rows(None, 2, 10, 10, p, None, 0, 0, out, None) != 0  # no logits
    assert lib.swl_agg_set_worker_sampling(-1, 1, 1.0, 0, 1.0) != 0
    assert "worker_id" in native.last_error()
    assert lib.swl_agg_set_sampling_seed(7) == 0
