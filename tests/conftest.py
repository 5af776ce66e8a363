import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, ROOT)
sys.path.insert(0, GOLDEN)
# dan's own host code (answer formatting) is installed beside this package: the offline
# install of the reference under baseline/_ref when present.
_DAN = os.path.join(ROOT, "baseline", "_ref")
if os.path.isdir(os.path.join(_DAN, "dan")):
    sys.path.append(_DAN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def golden(name):
    path = os.path.join(GOLDEN, name)
    if name.endswith(".json"):
        with open(path) as f:
            return json.load(f)
    import torch

    return torch.load(path, weights_only=True)


def plans_from_json(recs):
    from dan_b200.plan import Branch, ReadPlan

    return [ReadPlan(r["prefix"], branches=[Branch(b["suffix"], b["label_ids"]) for b in r["branches"]],
                     static=r["static"]) for r in recs]


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda:0")
