"""Shared pytest setup: the `gpu` marker, the package/oracle imports and fixtures."""
import importlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_package():
    """The product package (its directory name is not a Python identifier)."""
    return importlib.import_module("moebius-cpu_b200")


def load_oracle():
    from oracle import oracle
    return oracle


def load_golden(name):
    from safetensors.numpy import load_file
    return load_file(os.path.join(GOLDEN, name))


def scaled_err(got, want):
    """max |g − w| / (1 + |w|): the reference's assert_close metric (tests/kernels.rs:29-38)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    if got.size == 0:
        return 0.0
    return float(np.max(np.abs(got - want) / (1.0 + np.abs(want))))


def max_rel_err(got, want):
    """max |g − w| / max |w|: the per-kernel "max relative error" gate, normalised by the
    output's largest magnitude (outputs near zero carry only absolute error)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    if got.size == 0:
        return 0.0
    return float(np.max(np.abs(got - want)) / max(float(np.max(np.abs(want))), 1e-30))


def rel_l2(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.sqrt(np.sum((got - want) ** 2) / max(np.sum(want * want), 1e-300)))


@pytest.fixture(scope="session")
def oracle():
    return load_oracle()


@pytest.fixture(scope="session")
def mbx():
    return load_package()


@pytest.fixture(scope="session")
def ctx(mbx):
    c = mbx.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def ref_fixture():
    return load_golden("kernels_ref.safetensors")


@pytest.fixture(scope="session")
def extra_fixture():
    return load_golden("kernels_extra.safetensors")
