import glob
import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2 or more GPUs")


def fixture_names():
    return sorted(os.path.basename(p)[:-5] for p in glob.glob(os.path.join(GOLDEN, "*.json")) if not p.endswith("signs.json"))


class Fixture:
    def __init__(self, name):
        self.name = name
        self.meta = json.load(open(os.path.join(GOLDEN, name + ".json")))
        self.rows, self.K = self.meta["rows"], self.meta["K"]
        self.slot = np.fromfile(os.path.join(GOLDEN, name + ".slot"), np.uint8)
        self.x = np.load(os.path.join(GOLDEN, name + ".x.npy"))
        self.X = np.load(os.path.join(GOLDEN, name + ".X.npy"))
        self.y_ref = np.load(os.path.join(GOLDEN, name + ".y_ref.npy"))
        self.Y_ref = np.load(os.path.join(GOLDEN, name + ".Y_ref.npy"))


def load_fixture(name):
    return Fixture(name)


@pytest.fixture(params=fixture_names())
def golden(request):
    return Fixture(request.param)
