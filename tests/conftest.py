import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


# Run order: the kernel and engine parity suites first, then the
# multi-process and end-to-end integration tests and the newest suites, the
# no-allocation entry points last; file order within each group (a run that
# stops at its first failure then reports the core results first).
_LATE = ("test_shard_gpu.py", "test_worker_process_gpu.py", "test_donor_gpu.py", "test_checkpoint_gpu.py")
_LATE_TESTS = {"test_mixed_step_device_tokens_and_graph_replay", "test_subset_view_steps_only_its_slots",
               "test_profile_step_reports_the_reference_line",
               "test_config2_full_size_step_properties", "test_sampled_tokens_follow_the_reference_rule",
               "test_sampling_without_uniforms_is_seeded", "test_lm_head_round_samples_with_each_workers_state",
               "test_main_loop_serves_two_workers[sampling]"}
_LAST = ("test_zz_no_alloc.py",)


def pytest_collection_modifyitems(config, items):
    def key(item):
        name = Path(str(item.fspath)).name
        if name in _LAST:
            return (2, 0)
        if name in _LATE:
            return (1, 1 + _LATE.index(name))
        late = item.name in _LATE_TESTS or getattr(item, "originalname", item.name) in _LATE_TESTS
        return (1, 0) if late else (0, 0)
    items[:] = [it for _, it in sorted(enumerate(items), key=lambda p: (*key(p[1]), p[0]))]


@pytest.fixture
def scratch(request):
    """A fresh directory for one test's files inside the repository
    (tests/_scratch/<test>), removed afterwards."""
    import re
    import shutil
    d = ROOT / "tests" / "_scratch" / re.sub(r"[^A-Za-z0-9_.-]", "_", request.node.name)
    shutil.rmtree(d, ignore_errors=True)
    d.mkdir(parents=True)
    yield d
    shutil.rmtree(d, ignore_errors=True)


@pytest.fixture(scope="session")
def native():
    """The C-ABI library (built if missing)."""
    from swarmlora_b200 import build, _native
    if not _native.LIB_PATH.exists():
        build.build()
    return _native


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    torch.cuda.init()
    return torch.device("cuda:0")
