import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "flashengine.cpp_b200"), os.path.join(ROOT, "tests"),
          os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs the CUDA path")


@pytest.fixture
def parity_record(request):
    """record(label, result): append a parity test's error figures (max_abs,
    n_over_2e-3, max_abs_vs_f32, ...) as one JSON line to the file named by
    FE_PARITY_LOG, when that variable is set; a no-op otherwise."""
    path = os.environ.get("FE_PARITY_LOG")

    def record(label, result):
        if not path:
            return
        with open(path, "a") as f:
            f.write(json.dumps({"test": request.node.nodeid, "case": label, **result}) + "\n")

    return record
