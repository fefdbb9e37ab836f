"""GPU parity of the tensor-core prefix-hit prefill (prefill_tc.cu): chunks
of several query rows per sequence over bf16 K/V, against the CPU oracle
(src/nn/attention.cpp:128-239 restated) run on the same bf16-rounded K/V.
Q and the softmax weights enter the tensor cores as bf16, so the bound is
the bf16-storage tolerance: max |out - ref| <= 1e-2 * max |ref|; the
measured errors (printed, pytest -s) are 3-7e-3 (the full cfg3 prefill in
test_gpu_full_configs.py: median 3.3e-3, max 6.9e-3 over 256 sequences)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def run_case(s1kv, oracle, torch, Hq, Hkv, totals, qlens, seed, steps_decode=0):
    D, bs = 128, 16
    rng = np.random.default_rng(seed)
    need = sum((t + steps_decode + bs - 1) // bs for t in totals) + 4
    order = rng.permutation(need).astype(np.int32)
    pool = s1kv.Pool(1, Hkv, D, need, bs, dtype="bf16", initial_free_list=order)
    op = oracle.Pool(Hkv, D, need, bs, free_order=order)
    seqs = list(range(len(totals)))
    k = [rng.standard_normal((t, Hkv, D), dtype=np.float32) for t in totals]
    v = [rng.standard_normal((t, Hkv, D), dtype=np.float32) for t in totals]
    q = rng.standard_normal((sum(qlens), Hq, D), dtype=np.float32)
    with pool.batch(seqs, totals, qlens) as b:
        b.append(0, torch.from_numpy(np.concatenate(k)).cuda(), torch.from_numpy(np.concatenate(v)).cuda())
        out = b.attention(0, torch.from_numpy(q).cuda()).cpu().numpy()
    ref, r0 = [], 0
    for s, t, ql, kk, vv in zip(seqs, totals, qlens, k, v):
        assert op.append(s, oracle.bf16_round(kk), oracle.bf16_round(vv)) == 0
        ref.append(op.attention(s, q[r0:r0 + ql], Hq))
        r0 += ql
    for s in seqs:
        np.testing.assert_array_equal(pool.block_table(s), op.block_table(s))
    assert pool.check_device() == 0
    return out, np.concatenate(ref)


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (16, 2), (8, 8), (16, 8)])
def test_prefill_tc_matches_oracle(s1kv, oracle, cuda, Hq, Hkv):
    # prefix + suffix lengths: chunk boundaries, partial tiles, empty prefix,
    # a one-row sequence mixed in
    totals = [2050 + 64, 100, 33, 300 + 129, 1 + 1, 16 * 5]
    qlens = [64, 100, 33, 129, 1, 16]
    out, ref = run_case(s1kv, oracle, cuda, Hq, Hkv, totals, qlens, seed=Hq + Hkv)
    assert np.isfinite(out).all()
    err = rel_err(out, ref)
    print(f"prefill Hq {Hq} Hkv {Hkv}: rel err {err:.2e}")
    assert err <= TOL_BF16, err


def test_prefill_tc_long_prefix_many_sequences(s1kv, oracle, cuda):
    rng = np.random.default_rng(9)
    qlens = [int(x) for x in rng.integers(1, 300, size=12)]
    totals = [1500 + q for q in qlens]
    out, ref = run_case(s1kv, oracle, cuda, 32, 8, totals, qlens, seed=3)
    err = rel_err(out, ref)
    print(f"prefill, 12 sequences over a 1500-token prefix: rel err {err:.2e}")
    assert err <= TOL_BF16, err
