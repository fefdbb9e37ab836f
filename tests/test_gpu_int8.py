"""int8 projections on the GPU (s1kv_quantize_rows, s1kv_matmul_int8)
against the oracle (src/quantized_tensor.cpp restated) and the reference's
own outputs (tests/golden/int8.npz):
  * quantization is bit-exact: the int8 values and the per-row scales;
  * the product is within 2e-5 of the output scale (max |reference|) of the
    reference's sequential fp32 sum, and the same on every run;
  * shapes: the Qwen3-0.6B projections of the reference's model (hidden
    1024, q 2048, k/v 1024, MLP 3072; src/nn/attention.cpp:253-254,
    tests/test_layer.cpp:20-27), batches of 1-13 rows, odd widths, an
    all-zero weight row, K up to 4096 and the error for K beyond the limit."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "int8.npz")
TOL = 2e-5  # of max |reference output|


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def gpu_quantize(s1kv, torch, w):
    qt = s1kv.quantize_tensor(w)
    torch.cuda.synchronize()
    return qt, qt.data.cpu().numpy(), qt.scales.cpu().numpy()


def close(out, ref):
    scale = max(float(np.abs(ref).max()), 1e-30)
    err = float(np.abs(out.astype(np.float64) - ref.astype(np.float64)).max())
    return err <= TOL * scale, err / scale


@pytest.mark.gpu
def test_reference_fixtures(s1kv, cuda):
    torch = cuda
    d = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in d.files})
    for n in names:
        qt, q, sc = gpu_quantize(s1kv, torch, d[f"{n}/w"])
        assert np.array_equal(q, d[f"{n}/q"]), n
        assert np.array_equal(bits(sc), bits(d[f"{n}/scales"])), n
        out = s1kv.matmul_quantized(d[f"{n}/x"], qt).cpu().numpy()
        ok, rel = close(out, d[f"{n}/out"])
        assert ok, (n, rel)


@pytest.mark.gpu
def test_reference_known_answers(s1kv, cuda):
    # tests/test_quantized_tensor.cpp:5-49 through the Python mirror
    t = np.array([[1.0, -2.0, 0.5], [10.0, -20.0, 5.0]], np.float32)
    qt = s1kv.quantize_tensor(t)
    assert (qt.rows, qt.cols) == (2, 3)
    for r in range(2):
        for c in range(3):
            assert s1kv.dequantize(qt, r, c) == pytest.approx(float(t[r, c]), rel=0.02)
    qt = s1kv.quantize_tensor(np.array([[0.01, 0.02], [1.0, 2.0]], np.float32))
    assert float(qt.scales[0]) != pytest.approx(float(qt.scales[1]))
    assert s1kv.dequantize(qt, 0, 0) == pytest.approx(0.01, rel=0.02)
    qt = s1kv.quantize_tensor(np.zeros((1, 2), np.float32))
    assert s1kv.dequantize(qt, 0, 0) == 0.0 and s1kv.dequantize(qt, 0, 1) == 0.0


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 3), (1024, 2048), (3072, 1024), (33, 151), (5, 4099)])
def test_quantize_bit_exact(s1kv, oracle, cuda, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    w = (rng.standard_normal((rows, cols)) * rng.uniform(1e-3, 50.0, size=(rows, 1))).astype(np.float32)
    w[rows // 2] = 0.0
    if cols > 2:
        w[0, 1] = -np.abs(w[0]).max()  # the row maximum negative
    _, q, sc = gpu_quantize(s1kv, cuda, w)
    oq, osc = oracle.quantize_rows(w)
    assert np.array_equal(sc.view(np.uint32), osc.view(np.uint32))
    assert np.array_equal(q, oq)


SHAPES = [
    (1, 1024, 2048),  # q_proj of one decode token
    (1, 1024, 1024),  # k_proj / v_proj
    (1, 2048, 1024),  # o_proj
    (1, 1024, 3072),  # gate / up
    (1, 3072, 1024),  # down
    (4, 1024, 4096),
    (8, 2048, 1024),
    (13, 1024, 200),  # more rows than one launch slice
    (2, 5, 3),        # odd width: byte loads
    (1, 1, 1),
    (3, 4096, 64),
    (1, 100, 777),
]


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_matmul_matches_oracle(s1kv, oracle, cuda, M, K, N):
    torch = cuda
    rng = np.random.default_rng(M * 131 + K * 7 + N)
    w = (rng.standard_normal((K, N)) * rng.uniform(0.01, 3.0, size=(K, 1))).astype(np.float32)
    w[K // 3] = 0.0
    x = rng.standard_normal((M, K)).astype(np.float32)
    qt, q, sc = gpu_quantize(s1kv, torch, w)
    ref = oracle.matmul_int8(x, q, sc)
    out = s1kv.matmul_quantized(x, qt)
    out2 = s1kv.matmul_quantized(x, qt)
    o = out.cpu().numpy()
    ok, rel = close(o, ref)
    assert ok, rel
    assert np.array_equal(bits(o), bits(out2.cpu().numpy())), "not deterministic"


@pytest.mark.gpu
def test_matmul_k_limit(s1kv, cuda):
    torch = cuda
    K = 1 << 15
    qt = s1kv.QuantizedTensor(torch.zeros((K, 8), dtype=torch.int8, device="cuda"),
                              torch.ones(K, dtype=torch.float32, device="cuda"))
    with pytest.raises(s1kv.S1KVError) as e:
        s1kv.matmul_quantized(torch.zeros((1, K), device="cuda"), qt)
    assert e.value.status == s1kv.EINVAL


@pytest.mark.gpu
def test_matmul_empty(s1kv, cuda):
    torch = cuda
    qt = s1kv.QuantizedTensor(torch.zeros((16, 0), dtype=torch.int8, device="cuda"),
                              torch.ones(16, dtype=torch.float32, device="cuda"))
    out = s1kv.matmul_quantized(torch.zeros((2, 16), device="cuda"), qt)
    assert tuple(out.shape) == (2, 0)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 3, 8])
def test_group_equals_separate(s1kv, oracle, cuda, M):
    # q/k/v of self_attention_quantized (src/nn/attention.cpp:307-309) in one launch
    torch = cuda
    rng = np.random.default_rng(90 + M)
    K = 1024
    ws = [(rng.standard_normal((K, N)) * 0.05).astype(np.float32) for N in (2048, 1024, 1024)]
    x = rng.standard_normal((M, K)).astype(np.float32)
    qts = [s1kv.quantize_tensor(w) for w in ws]
    grouped = [o.cpu().numpy() for o in s1kv.matmul_quantized_group(x, qts)]
    for qt, g in zip(qts, grouped):
        sep = s1kv.matmul_quantized(x, qt).cpu().numpy()
        assert np.array_equal(bits(g), bits(sep))
        ref = oracle.matmul_int8(x, qt.data.cpu().numpy(), qt.scales.cpu().numpy())
        ok, rel = close(g, ref)
        assert ok, rel


@pytest.mark.gpu
def test_group_limits(s1kv, cuda):
    torch = cuda
    qt = s1kv.quantize_tensor(np.ones((16, 8), np.float32))
    with pytest.raises(s1kv.S1KVError) as e:
        s1kv.matmul_quantized_group(np.ones((1, 16), np.float32), [qt] * 5)
    assert e.value.status == s1kv.EINVAL
