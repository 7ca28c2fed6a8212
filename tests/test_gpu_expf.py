"""The device's softmax weight function equals glibc expf: on every fix-up
table entry, on a strided sweep over all non-positive floats, and on random
inputs of the form the sampler produces ((l - max_l) / T)."""
import os

import numpy as np
import pytest

import lal_b200 as L
import oracle
from lal_b200 import _build

pytestmark = pytest.mark.gpu

TABLE = os.path.join(os.path.dirname(_build.SO), "_gen", "expf_fixups.bin")


def check(x):
    y_dev = L.debug_expf(x)
    y_ref = oracle.expf(x)
    bad = np.nonzero(y_dev.view(np.uint32) != y_ref.view(np.uint32))[0]
    assert bad.size == 0, f"{bad.size} mismatches, e.g. x={x[bad[:5]]}"


def test_every_table_entry():
    raw = np.fromfile(TABLE, np.uint32)
    n = int(raw[0])
    check(raw[1:1 + n].view(np.float32).copy())


def test_strided_sweep_of_non_positive_floats():
    # every 61st bit pattern from -0 down to -inf: ~35M inputs
    bitsv = np.arange(0x80000000, 0xFF800001, 61, dtype=np.uint64).astype(np.uint32)
    for chunk in np.array_split(bitsv, 8):
        check(chunk.view(np.float32).copy())


def test_sampler_shaped_inputs():
    rng = np.random.default_rng(0)
    lg = (rng.standard_normal(2_000_000) * 4).astype(np.float32)
    mx = lg.max()
    for T in (0.5, 0.7, 0.8, 1.0, 1.3):
        x = ((lg - mx) / np.float32(T)).astype(np.float32)
        check(x)
