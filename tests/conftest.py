import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "nemo-c_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    # build what is missing (a fresh checkout has no .so files); the GPU box gets prebuilt copies
    lib = os.path.join(ROOT, "nemo-c_b200", "libnemoasr_b200.so")
    olib = os.path.join(ROOT, "oracle", "liboracle.so")
    if not os.path.exists(olib):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    if not os.path.exists(lib):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "nemo-c_b200")], check=True)


@pytest.fixture(scope="session")
def tiny_ckpt(tmp_path_factory):
    import nemoasr_b200 as nb
    d = str(tmp_path_factory.mktemp("ckpt_tiny"))
    nb.synth_write(d, nb.synth_tiny(seed=7))
    return d


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "golden_tiny.npz"))
