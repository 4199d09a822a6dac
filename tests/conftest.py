"""Shared pytest configuration.

`-m gpu` tests need a CUDA device and the built library; everything else
runs on CPU.  The oracle (`oracle/`) is importable from tests as
`ozaki_oracle`; it is the checker, never the thing measured.
"""

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def golden():
    with np.load(os.path.join(GOLDEN, "golden_cases.npz")) as z:
        arrays = {k: z[k] for k in z.files}
    with open(os.path.join(GOLDEN, "golden_meta.json")) as f:
        meta = json.load(f)
    return arrays, meta


def bf16_bits_to_f32(u16):
    return (np.asarray(u16, dtype=np.uint32) << 16).view(np.float32)


def same_bits(a, b):
    """Bitwise equality of float arrays, all NaNs counted equal."""
    a = np.asarray(a)
    b = np.asarray(b)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    ia = a.view(np.uint32 if a.dtype == np.float32 else np.uint64)
    ib = b.view(np.uint32 if b.dtype == np.float32 else np.uint64)
    return bool(np.all((ia == ib) | na))
