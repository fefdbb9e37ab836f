"""q/k RMSNorm + RoPE + append in one kernel (s1kv_batch_norm_rope_append)
against the oracle's reference chain rmsnorm -> apply_rope -> append
(src/nn/attention.cpp:316-322): the rotated q and the stored K bytes are
bit-exact (fp32 storage; bf16 storage = the exact fp32 value rounded), V
bytes are the input; for a step whose query rows are its appended tokens and
for one that mixes a prompt appended without queries with decode rows."""
import numpy as np
import pytest


def _chain(oracle, x, w, pos):
    return oracle.apply_rope(oracle.rmsnorm(x, w), pos=np.asarray(pos))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,D", [("f32", 128), ("bf16", 128), ("f32", 64)])
def test_norm_rope_append_matches_reference_chain(s1kv, oracle, cuda, dtype, D):
    import torch
    Hq, Hkv, bs = 16, 8, 16
    rng = np.random.default_rng(D + (dtype == "bf16"))
    pool = s1kv.Pool(1, Hkv, D, 64, bs, dtype=dtype)
    qw = rng.standard_normal(D).astype(np.float32)
    kw = rng.standard_normal(D).astype(np.float32)
    qw_d, kw_d = torch.from_numpy(qw).cuda(), torch.from_numpy(kw).cuda()
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    kst_of = lambda: pool.read_storage(0, 0)
    vst_of = lambda: pool.read_storage(0, 1)
    enc = (lambda a: a) if dtype == "f32" else oracle.to_bf16_bits

    # step 1: prefill of two sequences, query rows = appended tokens
    T = [7, 20]
    k = rng.standard_normal((sum(T), Hkv, D)).astype(np.float32) * 3
    v = rng.standard_normal((sum(T), Hkv, D)).astype(np.float32)
    q = rng.standard_normal((sum(T), Hq, D)).astype(np.float32) * 3
    with pool.batch([1, 2], T) as b:
        qo = b.norm_rope_append(0, cu(k), cu(v), kw_d, q=cu(q), q_norm_weight=qw_d).cpu().numpy()
    pos = np.concatenate([np.arange(t) for t in T])
    assert np.array_equal(qo, _chain(oracle, q, qw, pos))
    kst, vst = kst_of(), vst_of()
    off = 0
    for s, t in zip((1, 2), T):
        tab = pool.block_table(s)
        slots = [tab[i // bs] * bs + i % bs for i in range(t)]
        assert np.array_equal(kst[slots], enc(_chain(oracle, k[off:off + t], kw, np.arange(t))))
        assert np.array_equal(vst[slots], enc(v[off:off + t]))
        off += t

    # step 2: seq 3 appends a 5-token prompt without queries; seqs 1, 2 decode
    k2 = rng.standard_normal((7, Hkv, D)).astype(np.float32)
    v2 = rng.standard_normal((7, Hkv, D)).astype(np.float32)
    q2 = rng.standard_normal((2, Hq, D)).astype(np.float32)
    with pool.batch([1, 2, 3], [1, 1, 5], [1, 1, 0]) as b:
        qo2 = b.norm_rope_append(0, cu(k2), cu(v2), kw_d, q=cu(q2), q_norm_weight=qw_d).cpu().numpy()
    assert np.array_equal(qo2, _chain(oracle, q2, qw, [T[0], T[1]]))
    kst, vst = kst_of(), vst_of()
    tab = pool.block_table(3)
    slots = [tab[i // bs] * bs + i % bs for i in range(5)]
    assert np.array_equal(kst[slots], enc(_chain(oracle, k2[2:], kw, np.arange(5))))
    assert np.array_equal(vst[slots], enc(v2[2:]))
    for s, i in ((1, 0), (2, 1)):
        tab = pool.block_table(s)
        slot = tab[T[s - 1] // bs] * bs + T[s - 1] % bs
        assert np.array_equal(kst[slot], enc(_chain(oracle, k2[i:i + 1], kw, [T[s - 1]]))[0])
    assert pool.check_device() == 0
    pool.close()


@pytest.mark.gpu
def test_fused_norm_division_is_correctly_rounded(s1kv, cuda):
    """The normalisation divides each element by the row's rms with a
    reciprocal and one FMA correction; on 2^12 numerators x 2^11 divisors
    (random magnitudes over 2^-20 .. 2^20, both signs, zeros, rms-like values
    around 1e-3 .. 1e3) it equals the correctly rounded quotient bit for bit."""
    import torch
    rng = np.random.default_rng(99)
    xs = (rng.standard_normal(4096) * np.exp2(rng.uniform(-20, 20, 4096))).astype(np.float32)
    xs[:4] = [0.0, -0.0, 1.0, -3.0]
    ds = np.concatenate([np.exp2(rng.uniform(-10, 10, 1024)),
                         np.sqrt(rng.uniform(1e-6, 1e6, 1024))]).astype(np.float32)
    bad = torch.zeros(1, dtype=torch.int64, device="cuda")
    L = s1kv.lib()
    assert L.s1kv_debug_div_check(torch.from_numpy(xs).cuda().data_ptr(), xs.size, torch.from_numpy(ds).cuda().data_ptr(),
                                  ds.size, bad.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert int(bad.item()) == 0
