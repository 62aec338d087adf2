"""Shared test setup: markers, repository paths and golden-vector loading."""
import glob
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built native library")


def golden_fit_cases():
    return sorted(os.path.basename(p)[4:-4] for p in glob.glob(os.path.join(GOLDEN, "fit_*.npz")))


def load_golden(name):
    return np.load(os.path.join(GOLDEN, name))


def load_layouts():
    with open(os.path.join(GOLDEN, "layouts.json")) as fh:
        return json.load(fh)


@pytest.fixture(autouse=True)
def _skip_gpu_without_cuda(request):
    if request.node.get_closest_marker("gpu") is not None:
        import torch
        if not torch.cuda.is_available():
            pytest.skip("CUDA device required")
