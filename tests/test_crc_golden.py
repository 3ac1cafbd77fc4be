"""The per-row CRC32 files that pin the benchmark-shape integer GEMMs
(tests/golden/make_crc.py) agree with the oracle: a few rows recomputed on
the CPU, first, last and in between."""
import sys

import numpy as np
import pytest

from conftest import GOLDEN


@pytest.mark.parametrize("kind", ["u8s8", "hmx"])
def test_crc_rows_match_oracle(oracle, kind):
    if str(GOLDEN) not in sys.path:
        sys.path.insert(0, str(GOLDEN))
    import make_crc
    d = make_crc.inputs(kind)
    crcs = np.load(make_crc.FILES[kind])
    assert crcs.shape == (make_crc.M,) and crcs.dtype == np.uint32
    for r in (0, 1, 8191, make_crc.M - 1):
        got = make_crc.row_crcs(make_crc.oracle_rows(kind, d, r, r + 1))
        assert got[0] == crcs[r], (kind, r)
