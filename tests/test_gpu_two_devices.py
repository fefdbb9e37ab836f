"""One process driving two GPUs: kernel attributes (dynamic shared memory,
cluster size) are per device, so the decode kernels (fp32 and bf16 K/V) and
the int8 product must work on device 1 after device 0 has run them.
Skipped with fewer than two GPUs."""
import numpy as np
import pytest


def _decode_on(s1kv, oracle, torch, dev, dtype):
    rng = np.random.default_rng(3 + dev)
    Hq, Hkv, D, bs = 32, 8, 128, 16
    ctx = [130, 777, 2048]
    seqs = [1, 2, 3]
    pool = s1kv.Pool(1, Hkv, D, 400, bs, dtype=dtype, device=dev)
    opool = oracle.Pool(Hkv, D, 400, bs)
    ks = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    vs = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    if dtype == "bf16":
        ks = [oracle.bf16_round(k) for k in ks]
        vs = [oracle.bf16_round(v) for v in vs]
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda(dev)
    with pool.batch(seqs, ctx, [0] * len(ctx)) as b:
        b.append(0, cu(np.concatenate(ks)), cu(np.concatenate(vs)))
    for s, k, v in zip(seqs, ks, vs):
        opool.append(s, k, v)
    q = rng.standard_normal((len(seqs), Hq, D), dtype=np.float32)
    with pool.batch(seqs, [0] * len(seqs), [1] * len(seqs)) as b:
        out = b.attention(0, cu(q)).cpu().numpy()
    ref = np.concatenate([opool.attention(s, q[i:i + 1], Hq) for i, s in enumerate(seqs)])
    err = float(np.abs(out - ref).max() / np.abs(ref).max())
    assert err <= 2e-5, (dev, dtype, err)
    assert pool.check_device() == 0
    pool.close()


@pytest.mark.gpu
def test_two_devices_in_one_process(s1kv, oracle, cuda):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    for dev in (0, 1):
        with torch.cuda.device(dev):
            for dtype in ("f32", "bf16"):
                _decode_on(s1kv, oracle, torch, dev, dtype)
            rng = np.random.default_rng(50 + dev)
            w = (rng.standard_normal((3072, 1024)) * 0.05).astype(np.float32)
            x = rng.standard_normal((8, 3072)).astype(np.float32)
            qt = s1kv.quantize_tensor(w, device=dev)
            out = s1kv.matmul_quantized(x, qt).cpu().numpy()
            ref = oracle.matmul_int8(x, qt.data.cpu().numpy(), qt.scales.cpu().numpy())
            assert float(np.abs(out - ref).max()) <= 2e-5 * float(np.abs(ref).max()), dev
