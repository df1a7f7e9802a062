import functools
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    """The reference's CPU path built from its sources; skipped where it was never built."""
    from oracle.oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/libref_moe.so not built (reference sources absent)")
    return Reference(1)


@functools.lru_cache(maxsize=None)
def cached_layer(D, E, K, I, layer=0, zipf=None, down_type=12):
    from laii_b200 import synth
    L = synth.make_moe_layer(D, E, K, I, layer=layer, down_type=down_type)
    if zipf is not None:
        L.bias = synth.zipf_bias(L, s=zipf)
    return L


@functools.lru_cache(maxsize=None)
def cached_dense(D, I, layer=0):
    from laii_b200 import synth
    return synth.make_dense_layer(D, I, layer=layer)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
