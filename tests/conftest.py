import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "vestra-kernels_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the C-ABI library)")


def xorshift32_values(n: int, seed: int, centred: bool = True):
    """The xorshift32 generator of tests/attention_matches_naive.rs:5-16 and
    src/attention.rs:240-249: (state / u32::MAX) * 2 - 1, all in f32."""
    import numpy as np

    out = np.empty(n, np.float32)
    s = seed & 0xFFFFFFFF
    inv = np.float32(4294967295.0)
    for i in range(n):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        v = np.float32(s) / inv
        out[i] = v * np.float32(2.0) - np.float32(1.0) if centred else v - np.float32(0.5)
    return out


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle

    oracle.lib()
    return oracle
