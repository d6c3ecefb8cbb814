"""CPU tests: the Page16 oracle against golden vectors of the reference's own
Triton kernel (core/page16_native.py:17-80, run by Triton's interpreter)."""
import numpy as np
import pytest

from oracle.page16 import lse_merge_reference, page16_decode_reference
from tests.golden.inputs import PAGE16_CASES, checksum, page16_case

GOLDEN = __import__("pathlib").Path(__file__).parent / "golden"


@pytest.mark.parametrize("name", sorted(PAGE16_CASES))
def test_oracle_matches_reference_triton(name):
    cfg = PAGE16_CASES[name]
    q, k, v, bt, lens = page16_case(**cfg)
    g = np.load(GOLDEN / f"page16_{name}.npz")
    assert str(g["inputs_sha"]) == checksum(q, k, v, bt, lens), "seeded inputs drifted"
    out = page16_decode_reference(q, k, v, bt, lens, float(g["scale"]), int(g["n_rep"]))
    ref = g["out"]
    # fp32 reference outputs: 1e-5; fp16 outputs are rounded to fp16 by the reference
    tol = 1e-5 if q.dtype == np.float32 else 1e-3
    assert np.max(np.abs(out - ref)) < tol


def test_oracle_empty_request_is_nan():
    q, k, v, bt, lens = page16_case(seed=9, batch=2, hq=4, hkv=2, d=16, lens=(0, 20), num_pages=8)
    out = page16_decode_reference(q, k, v, bt, lens, 0.25, 2)
    assert np.isnan(out[0]).all() and np.isfinite(out[1]).all()


def test_lse_merge_equals_unsplit():
    q, k, v, bt, lens = page16_case(seed=4, batch=1, hq=4, hkv=2, d=16, lens=(160,), num_pages=10)
    full, lse = page16_decode_reference(q, k, v, bt, lens, 0.25, 2, return_lse=True)
    parts, lses = [], []
    for lo, hi in [(0, 3), (3, 7), (7, 10)]:
        o, l = page16_decode_reference(q, k, v, bt[:, lo:hi], np.array([16 * (hi - lo)], np.int32), 0.25, 2,
                                       return_lse=True)
        parts.append(o[0])
        lses.append(l[0])
    m, ml = lse_merge_reference(np.stack(parts), np.stack(lses))
    assert np.allclose(m, full[0], atol=1e-12) and np.allclose(ml, lse[0], atol=1e-12)
