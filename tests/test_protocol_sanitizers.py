"""Race and memory checking of the host protocol on the CPU: the aggregator's
main loop (swarmlora_b200/csrc/agg_protocol.h, the code the library runs
around its GPU rounds) and the worker-side queue
(swarmlora_b200/csrc/ipc_queue.cpp), driven by tests/native/protocol_stress.cpp
(ten worker threads joining and leaving at different times, a stalled slot
evicted by the barrier timeout, a foreign command evicted by validation;
the same with every round's epoch stored late by another thread, as the
device stores it in the library's deferred completion; then worker processes, one killed by SIGKILL mid-token as the reference's
fault driver does, evicted while the others finish), built and run under
ThreadSanitizer and under AddressSanitizer with UBSan.
The reference has no race detection for this path (its ownership checks run
at run time only)."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _cuda_include():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    inc = Path(nvcc).resolve().parent.parent / "include"
    return inc if (inc / "cuda_runtime.h").exists() else Path("/usr/local/cuda/include")


@pytest.mark.parametrize("sanitizer", ["thread", "address,undefined"])
def test_protocol_stress_under_sanitizer(scratch, sanitizer):
    exe = scratch / "protocol_stress"
    cmd = ["g++", "-std=c++17", "-O1", "-g", f"-fsanitize={sanitizer}", "-pthread",
           f"-I{ROOT / 'swarmlora_b200' / 'csrc'}", f"-I{ROOT / 'include'}", f"-I{_cuda_include()}",
           str(ROOT / "tests" / "native" / "protocol_stress.cpp"),
           str(ROOT / "swarmlora_b200" / "csrc" / "ipc_queue.cpp"), "-o", str(exe), "-lrt"]
    # thread fences are not modelled by the thread sanitizer; the one in
    # swl_q_create runs before any other thread exists
    cmd.insert(1, "-Wno-tsan" if sanitizer == "thread" else "-fno-sanitize-recover=undefined")
    build = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert build.returncode == 0, build.stderr[-4000:]
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1", UBSAN_OPTIONS="print_stacktrace=1")
    # threads; the same with each round's epoch stored late by another thread
    # (the device-published completion); then forked worker processes, one of
    # them killed by SIGKILL mid-token (the reference's fault driver), evicted
    # while the rest finish
    for mode in ([], ["--deferred"], ["--processes"]):
        run = subprocess.run([str(exe), *mode], capture_output=True, text=True, timeout=300, env=env)
        out = run.stdout + run.stderr
        assert run.returncode == 0 and "protocol stress ok" in run.stdout, out[-6000:]
        for marker in ("ThreadSanitizer", "AddressSanitizer", "LeakSanitizer", "runtime error"):
            assert marker not in run.stderr, out[-6000:]
        if mode == ["--processes"]:
            assert "1 killed and evicted" in run.stdout
        if mode == ["--deferred"]:
            assert "epochs published by a deferred publisher" in run.stdout
