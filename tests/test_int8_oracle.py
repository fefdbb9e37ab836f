"""Pins the oracle's int8 projection restatement (oracle/kvoracle.c:
kvo_quantize_rows, kvo_matmul_int8) before the GPU is checked against it:
  * the known answers of the reference's own tests/test_quantized_tensor.cpp,
  * bit for bit against the committed fixtures tests/golden/int8.npz, which
    the reference's quantize_tensor / matmul_quantized produced
    (tests/golden/make_golden.py),
  * and, where the reference was compiled here (oracle/_ref), bit for bit
    against it on fresh seeded inputs, single-threaded and over its
    ThreadPool."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "int8.npz")


def cases():
    d = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in d.files})
    return d, names


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_quantize_recovers_values(oracle):
    # tests/test_quantized_tensor.cpp:5-23
    t = np.array([[1.0, -2.0, 0.5], [10.0, -20.0, 5.0]], np.float32)
    q, sc = oracle.quantize_rows(t)
    assert q.shape == (2, 3)
    rec = q.astype(np.float32) * sc[:, None]
    np.testing.assert_allclose(rec, t, rtol=0.02)


def test_each_row_own_scale(oracle):
    # tests/test_quantized_tensor.cpp:25-39
    q, sc = oracle.quantize_rows(np.array([[0.01, 0.02], [1.0, 2.0]], np.float32))
    assert sc[0] != pytest.approx(sc[1])
    assert float(q[0, 0]) * sc[0] == pytest.approx(0.01, rel=0.02)
    assert float(q[0, 1]) * sc[0] == pytest.approx(0.02, rel=0.02)


def test_zero_row_no_nan(oracle):
    # tests/test_quantized_tensor.cpp:41-49
    q, sc = oracle.quantize_rows(np.zeros((1, 2), np.float32))
    assert sc[0] == 1.0 and not np.isnan(sc).any()
    assert (q == 0).all()


def test_blocked_matmul_close_to_float(oracle):
    # tests/test_quantized_tensor.cpp:51-75: within 5% of max|float matmul|
    d = np.load(GOLDEN)
    a, b = d["kat_blocked/x"], d["kat_blocked/w"]
    q, sc = oracle.quantize_rows(b)
    out = oracle.matmul_int8(a, q, sc)
    ref = (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)
    assert np.abs(out.astype(np.float64) - ref).max() < 0.05 * np.abs(ref).max()


def test_oracle_matches_reference_fixtures(oracle):
    d, names = cases()
    assert len(names) >= 7
    for n in names:
        q, sc = oracle.quantize_rows(d[f"{n}/w"])
        assert np.array_equal(q, d[f"{n}/q"]), n
        assert np.array_equal(bits(sc), bits(d[f"{n}/scales"])), n
        out = oracle.matmul_int8(d[f"{n}/x"], q, sc)
        assert np.array_equal(bits(out), bits(d[f"{n}/out"])), n


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                                    "oracle", "_ref", "libs1ref.so")),
                    reason="reference not compiled here")
@pytest.mark.parametrize("M,K,N", [(1, 1024, 600), (4, 300, 17), (2, 33, 520)])
def test_oracle_matches_reference_fresh(oracle, M, K, N):
    rng = np.random.default_rng(M * 1000 + K + N)
    w = (rng.standard_normal((K, N)) * 0.3).astype(np.float32)
    w[::7] *= 40.0
    w[3] = 0.0
    x = rng.standard_normal((M, K)).astype(np.float32)
    q, sc = oracle.quantize_rows(w)
    rq, rsc = oracle.ref_quantize_rows(w)
    assert np.array_equal(q, rq) and np.array_equal(bits(sc), bits(rsc))
    out = oracle.matmul_int8(x, q, sc)
    assert np.array_equal(bits(out), bits(oracle.ref_matmul_int8(x, q, sc)))
    assert np.array_equal(bits(out), bits(oracle.ref_matmul_int8(x, q, sc, threaded=True)))
