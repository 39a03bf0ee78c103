import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def built_lib():
    from wisp_b200 import build
    return build.build()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from wisp_b200 import build
    build.build()
    return torch.device("cuda:0")


GOLDEN = ROOT / "tests" / "golden"


@pytest.fixture(scope="session")
def golden():
    import json
    import numpy as np
    meta = json.loads((GOLDEN / "golden.json").read_text())
    arrays = dict(np.load(GOLDEN / "golden_outputs.npz"))
    return meta, arrays


def shape_of(spec):
    from wisp_b200 import converter as cv
    return cv.MoEShape(**spec["shape"])


@pytest.fixture(scope="session")
def golden_dirs(golden, tmp_path_factory):
    """The golden models rewritten by wisp_b200.converter (must hash-match the
    reference-written blobs)."""
    from wisp_b200 import converter as cv
    meta, _ = golden
    out = {}
    for name, spec in meta["models"].items():
        d = tmp_path_factory.mktemp(name)
        cv.write_model_dir(d, shape_of(spec), spec["seed"], router_bias=(spec["bias"] == "random"),
                           zipf_s=1.1 if spec["bias"] == "zipf" else None)
        out[name] = d
    return out
