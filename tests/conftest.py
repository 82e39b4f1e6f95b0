import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "supra2-img-web_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run on the GPU box")


class Golden:
    """The golden vectors in tests/golden (reference dump format, tools/reference.py:41-54)."""

    def __init__(self, root=GOLDEN):
        self.root = root
        with open(os.path.join(root, "index.json")) as f:
            self.index = json.load(f)

    def __call__(self, name):
        meta = self.index["tensors"][name]
        a = np.fromfile(os.path.join(self.root, name + ".bin"), dtype="<f4")
        return a.reshape(meta["shape"])

    def meta(self, name):
        return self.index["tensors"][name]

    @property
    def cases(self):
        return self.index["cases"]


@pytest.fixture(scope="session")
def golden():
    return Golden()


@pytest.fixture(scope="session")
def gpu():
    """One libsupra_attn context on cuda:0, running on torch's current stream."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import supra_attn

    g = supra_attn.GPU(0, stream=torch.cuda.current_stream())
    yield g
    g.close()
