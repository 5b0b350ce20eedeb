import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden")
# The reference tree (read only, never needed on a GPU box): $REF_ROOT, else a
# directory `reference` beside this repository's root.  Tests that read it skip
# when it is absent.
REF_ROOT = os.environ.get("REF_ROOT") or os.path.abspath(os.path.join(ROOT, "..", "reference"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


def pkg():
    return importlib.import_module("embeddinggemma2-amdkfd_b200")


@pytest.fixture(scope="session")
def eg2():
    return pkg()


@pytest.fixture(scope="session")
def syn():
    return importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")


@pytest.fixture(scope="session")
def model_baseline(syn):
    return syn.model_path(1234, "baseline")


@pytest.fixture(scope="session")
def model_plus1(syn):
    return syn.model_path(1234, "plus1")


@pytest.fixture(scope="session")
def port():
    import oracle
    oracle.build(ref=False)
    return oracle.Port()


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, name), allow_pickle=False))


def cosine(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return (a * b).sum(-1) / np.sqrt((a * a).sum(-1) * (b * b).sum(-1))
