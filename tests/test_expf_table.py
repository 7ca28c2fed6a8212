"""The glibc-expf fix-up table embedded in liblal_tail.so: generated at build
time by calling this host's glibc expf on every non-positive float.  Here
every entry is re-checked against glibc expf, so a host whose libm picks a
different expf variant is noticed."""
import os

import numpy as np
import pytest

import oracle
from lal_b200 import _build

TABLE = os.path.join(os.path.dirname(_build.SO), "_gen", "expf_fixups.bin")


@pytest.fixture(scope="module")
def table():
    if not os.path.exists(TABLE):
        _build.build_expf_table()
    raw = np.fromfile(TABLE, np.uint32)
    n = int(raw[0])
    assert raw.size == 1 + 2 * n
    return raw[1:1 + n], raw[1 + n:]


def test_table_is_sorted_and_plausible(table):
    x, y = table
    assert 10_000 < x.size < 1_000_000
    assert np.all(np.diff(x.astype(np.int64)) > 0)
    assert np.all(x >= 0x80000000)          # non-positive inputs only


def test_table_entries_are_glibc_results(table):
    x, y = table
    g = oracle.expf(x.view(np.float32))
    np.testing.assert_array_equal(g.view(np.uint32), y)
    # and each entry is a 1-ulp correction of the once-rounded exp
    xd = x.view(np.float32).astype(np.float64)
    approx = np.exp(xd).astype(np.float32)
    diff = np.abs(approx.view(np.int32).astype(np.int64) - y.view(np.int32).astype(np.int64))
    assert np.mean(diff <= 1) > 0.999
