"""Pins the CPU oracle (oracle/kvoracle.c) before anything is checked
against it:
  * against the known answers in the reference's own tests
    (tests/test_rope.cpp, tests/test_attention.cpp, tests/test_kv_block_pool.cpp),
  * against the committed golden fixtures, produced by the reference's own
    code (tests/golden/make_golden.py),
  * and, where the reference was compiled here (oracle/_ref), bit for bit
    against it on fresh seeded inputs."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import scenarios as S  # noqa: E402

GOLDEN = os.path.join(HERE, "golden")


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# ------------------------------------------------ reference known answers --

def test_rope_position_zero_is_identity(oracle):
    # tests/test_rope.cpp:5-18
    x = np.array([[1.0, 2.0, 3.0, 4.0]], np.float32)
    np.testing.assert_allclose(oracle.apply_rope(x, 0), x, rtol=1e-6)


def test_rope_position_one_hand_rotation(oracle):
    # tests/test_rope.cpp:20-34: [1,0,1,0] at pos 1 -> [-0.30117, 0, 1.38177, 0]
    out = oracle.apply_rope(np.array([[1.0, 0.0, 1.0, 0.0]], np.float32), 1)[0]
    assert out[0] == pytest.approx(-0.30117, rel=1e-3)
    assert out[1] == pytest.approx(0.0, abs=1e-3)
    assert out[2] == pytest.approx(1.38177, rel=1e-3)
    assert out[3] == pytest.approx(0.0, abs=1e-3)


def test_causal_mask_known_answer(oracle):
    # tests/test_attention.cpp:29-64
    Q = np.ones((2, 2, 2), np.float32)
    K = np.array([1, 0, 1, 0], np.float32).reshape(2, 1, 2)
    V = np.array([2, 4, 6, 8], np.float32).reshape(2, 1, 2)
    out = oracle.gqa_attention(Q, K, V, 2, 1, 2)
    np.testing.assert_allclose(out[0], [[2, 4], [2, 4]], rtol=1e-6)
    np.testing.assert_allclose(out[1], [[4, 6], [4, 6]], rtol=1e-6)


def test_paged_matches_contiguous_on_scattered_blocks(oracle):
    # tests/test_attention.cpp:66-120: blocks [3, 1, 0] via filler/remove
    p = oracle.Pool(1, 2, 4, 2)
    filler = np.zeros((2, 1, 2), np.float32)
    p.append(1, filler, filler)
    p.append(2, filler, filler)
    p.remove(1)
    K = np.array([1, -1, 2, -2, 3, -3, 4, -4, 5, -5], np.float32).reshape(5, 1, 2)
    V = np.array([10, 100, 20, 200, 30, 300, 40, 400, 50, 500], np.float32).reshape(5, 1, 2)
    p.append(0, K, V)
    assert list(p.block_table(0)) == [3, 1, 0]
    Q = (np.arange(1, 21, dtype=np.float32) / 10).reshape(5, 2, 2)
    expected = oracle.gqa_attention(Q, p.get_k(0), p.get_v(0), 2, 1, 2)
    np.testing.assert_allclose(p.attention(0, Q, 2), expected, rtol=1e-6)


def _t(vals):
    return np.asarray(vals, np.float32).reshape(len(vals), 1, 1)


def test_kv_block_pool_reference_cases(oracle):
    # tests/test_kv_block_pool.cpp:6-207, case by case
    p = oracle.Pool(1, 2, 4, 4)
    k = np.arange(1, 7, dtype=np.float32).reshape(3, 1, 2)
    v = k * 10
    assert p.append(0, k, v) == 0
    np.testing.assert_array_equal(p.get_k(0), k)
    np.testing.assert_array_equal(p.get_v(0), v)

    p = oracle.Pool(1, 1, 4, 2)  # 5 tokens over 3 blocks
    p.append(0, _t([1, 2, 3, 4, 5]), _t([10, 20, 30, 40, 50]))
    np.testing.assert_array_equal(p.get_k(0).ravel(), [1, 2, 3, 4, 5])

    p = oracle.Pool(1, 1, 4, 4)  # partial block continued across calls
    p.append(0, _t([1, 2, 3]), _t([1, 2, 3]))
    p.append(0, _t([4, 5, 6]), _t([4, 5, 6]))
    np.testing.assert_array_equal(p.get_k(0).ravel(), [1, 2, 3, 4, 5, 6])

    p = oracle.Pool(1, 1, 1, 2)  # remove frees for reuse; exhaustion errors
    p.append(0, _t([1, 2]), _t([1, 2]))
    assert p.append(1, _t([1, 2]), _t([1, 2])) == oracle.ENOBLOCKS
    p.remove(0)
    assert p.append(1, _t([1, 2]), _t([1, 2])) == 0
    np.testing.assert_array_equal(p.get_k(1).ravel(), [1, 2])
    with pytest.raises(RuntimeError):
        p.get_k(0)

    p = oracle.Pool(1, 1, 4, 2)
    with pytest.raises(RuntimeError):
        p.get_k(99)
    assert p.length(0) == 0
    p.append(0, _t([1, 2, 3]), _t([1, 2, 3]))
    assert p.length(0) == 3

    p = oracle.Pool(1, 1, 4, 4)  # truncate mid-block then append
    p.append(0, _t(range(1, 11)), _t(range(1, 11)))
    p.truncate(0, 5)
    assert p.length(0) == 5
    p.append(0, _t([100, 101]), _t([100, 101]))
    np.testing.assert_array_equal(p.get_k(0).ravel(), [1, 2, 3, 4, 5, 100, 101])

    p = oracle.Pool(1, 1, 4, 4)  # truncate at a block multiple frees one block
    p.append(0, _t(range(1, 11)), _t(range(1, 11)))
    p.truncate(0, 8)
    assert p.length(0) == 8 and p.num_free() == 2
    assert p.append(1, _t([1, 2, 3, 4, 5]), _t([1, 2, 3, 4, 5])) == 0

    p = oracle.Pool(1, 1, 4, 4)  # truncate no-op
    p.append(0, _t([1, 2, 3]), _t([1, 2, 3]))
    p.truncate(0, 10)
    p.truncate(0, 3)
    assert p.length(0) == 3

    p = oracle.Pool(1, 1, 4, 4)  # truncate to 0 keeps the sequence
    p.append(0, _t([1, 2, 3, 4]), _t([1, 2, 3, 4]))
    p.truncate(0, 0)
    assert p.length(0) == 0 and p.has(0)
    assert p.append(1, _t([9.0] * 16), _t([9.0] * 16)) == 0


# ------------------------------------------------------- golden fixtures --

def test_rope_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "rope.npz"))
    for D in (4, 64, 128):
        for pos in (0, 1, 4095, 131071):
            assert np.array_equal(bits(oracle.apply_rope(g[f"x_{D}"], pos)), bits(g[f"out_{D}_{pos}"])), (D, pos)


def run_pool_ops(pool, ops, seed, append):
    rng = np.random.default_rng(100 + seed)
    status, lengths, tables = [], [], []
    for kind, seq, n in ops:
        if kind == 0:
            k = rng.standard_normal((n, 1, 2), dtype=np.float32)
            st = append(pool, seq, k)
        elif kind == 1:
            st = pool.truncate(seq, n)
        else:
            st = pool.remove(seq)
        status.append(1 if st else 0)
        lengths.append(pool.length(seq))
        t = pool.block_table(seq)
        tables.append(-np.ones(12, np.int32) if t is None else np.pad(t, (0, 12 - len(t)), constant_values=-2))
    return np.array(status), np.array(lengths), np.stack(tables)


def test_pool_ops_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "pool_ops.npz"))
    for seed in range(4):
        ops = [tuple(int(x) for x in r) for r in g[f"ops_{seed}"]]
        st, ln, tb = run_pool_ops(oracle.Pool(1, 2, 12, 4), ops, seed, lambda p, s, k: p.append(s, k, k))
        np.testing.assert_array_equal(st, g[f"status_{seed}"])
        np.testing.assert_array_equal(ln, g[f"length_{seed}"])
        np.testing.assert_array_equal(tb, g[f"tables_{seed}"])


class OracleBackend:
    def new_pools(self, layers, H, D, max_blocks, bs, order):
        self.pools = [_oracle().Pool(H, D, max_blocks, bs, free_order=order) for _ in range(layers)]

    def rope(self, x, pos):
        return _oracle().apply_rope(x, pos)

    def append(self, layer, seq, k, v):
        assert self.pools[layer].append(seq, k, v) == 0

    def attention(self, layer, seq, q, Hq):
        return self.pools[layer].attention(seq, q, Hq)

    def length(self, seq, layer=0):
        return self.pools[layer].length(seq)

    def table(self, seq):
        return self.pools[0].block_table(seq)


def _oracle():
    from oracle import oracle as O
    return O


@pytest.mark.parametrize("name", list(S.SCENARIOS))
def test_scenarios_golden_bit_exact(oracle, name):
    g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    got = S.flatten(S.run_scenario(name, OracleBackend()), name)
    assert set(got) == set(g.files)
    for key in g.files:
        if key.startswith("table"):
            np.testing.assert_array_equal(got[key], g[key], err_msg=key)
        else:
            assert np.array_equal(bits(got[key]), bits(g[key])), key


# ------------------------------------------ against the compiled reference --

needs_ref = pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(HERE), "oracle", "_ref", "libs1ref.so")),
                               reason="reference not compiled here (oracle/_ref)")


@needs_ref
@pytest.mark.parametrize("seed", range(6))
def test_restatement_matches_reference_attention(oracle, seed):
    rng = np.random.default_rng(1000 + seed)
    Hkv = int(rng.choice([1, 2, 4]))
    G = int(rng.choice([1, 2, 3, 7]))
    D = int(rng.choice([2, 8, 64]))
    bs = int(rng.choice([1, 3, 16]))
    T = int(rng.integers(1, 90))
    q_len = int(rng.integers(1, T + 1))
    k = rng.standard_normal((T, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, D), dtype=np.float32)
    q = rng.standard_normal((q_len, G * Hkv, D), dtype=np.float32)
    nb = (T + bs - 1) // bs + 3
    rp, op = oracle.RefPool(Hkv, D, nb, bs), oracle.Pool(Hkv, D, nb, bs)
    assert rp.append(9, k, v) == 0 and op.append(9, k, v) == 0
    np.testing.assert_array_equal(rp.block_table(9), op.block_table(9))
    assert np.array_equal(bits(rp.attention(9, q, G * Hkv)), bits(op.attention(9, q, G * Hkv)))
    assert np.array_equal(bits(oracle.ref_gqa_attention(q, k, v, G * Hkv, Hkv, D)),
                          bits(oracle.gqa_attention(q, k, v, G * Hkv, Hkv, D)))


@needs_ref
@pytest.mark.parametrize("D", [2, 6, 64, 128])
def test_restatement_matches_reference_rope(oracle, D):
    rng = np.random.default_rng(D)
    x = rng.standard_normal((17, 3, D), dtype=np.float32)
    for pos in (0, 7, 1000, 65535, 131072 + 5):
        assert np.array_equal(bits(oracle.apply_rope(x, pos)), bits(oracle.ref_apply_rope(x, pos)))


@needs_ref
@pytest.mark.parametrize("seed", range(8))
def test_restatement_matches_reference_pool_ops(oracle, seed):
    ops = [({"append": 0, "truncate": 1, "remove": 2}[k], s, n) for k, s, n in S.pool_ops(50 + seed, n_ops=120)]
    ref = run_pool_ops(oracle.RefPool(1, 2, 12, 4), ops, seed, lambda p, s, k: p.append(s, k, k))
    mine = run_pool_ops(oracle.Pool(1, 2, 12, 4), ops, seed, lambda p, s, k: p.append(s, k, k))
    for a, b in zip(ref, mine):
        np.testing.assert_array_equal(a, b)


@needs_ref
def test_free_order_matches_remove_trick(oracle):
    """The explicit initial free list equals the reference's remove-trick
    free list: both pools allocate the same blocks afterwards."""
    order = np.random.default_rng(5).permutation(10).astype(np.int32)
    rp = oracle.RefPool(1, 1, 10, 2)
    z = np.zeros((2, 1, 1), np.float32)
    for i in range(10):
        rp.append(S.DUMMY_BASE + i, z, z)
    for i in S.remove_trick_plan(10, order):
        rp.remove(S.DUMMY_BASE + i)
    op = oracle.Pool(1, 1, 10, 2, free_order=order)
    k = np.ones((19, 1, 1), np.float32)
    rp.append(3, k, k)
    op.append(3, k, k)
    np.testing.assert_array_equal(rp.block_table(3), op.block_table(3))
    np.testing.assert_array_equal(op.block_table(3), order[::-1])


# ------------------------------------------------ sharing semantics (new) --

def test_fork_cow_refcounts(oracle):
    p = oracle.Pool(1, 2, 8, 4)
    k = np.arange(10 * 2, dtype=np.float32).reshape(10, 1, 2)
    p.append(0, k, k)                       # blocks 7, 6, 5 (2 tokens in the tail)
    assert p.fork(0, 1, 10) == 0
    t0 = p.block_table(0)
    assert list(p.block_table(1)) == list(t0)
    assert [p.refcount(b) for b in t0] == [2, 2, 2]
    rc, slots, (cs, cd) = p.reserve(1, 1)   # first write into the shared tail
    assert rc == 0 and cs == t0[-1] and cd == 4
    assert list(p.block_table(1)) == [t0[0], t0[1], 4]
    assert p.refcount(t0[-1]) == 1 and p.refcount(4) == 1
    np.testing.assert_array_equal(p.get_k(1)[:10], k)  # the copy carried the tail
    assert slots[0] == 4 * 4 + 2
    p.remove(0)                              # shared full blocks survive
    assert p.refcount(t0[0]) == 1 and p.refcount(t0[-1]) == 0
    assert list(p.free_list()[-1:]) == [t0[-1]]


def test_prefix_cache_lru(oracle):
    p = oracle.Pool(1, 1, 6, 2)
    toks = np.arange(7, dtype=np.int32)
    k = np.ones((7, 1, 1), np.float32)
    p.append(0, k, k)                        # blocks 5, 4, 3, 2 (last partial)
    assert p.prefix_insert(0, toks) == 3     # three full blocks registered
    p.remove(0)
    assert list(p.lru_list()) == [5, 4, 3] and list(p.free_list()) == [0, 1, 2]
    rc, hit = p.prefix_match(1, toks[:5])
    assert rc == 0 and hit == 4 and list(p.block_table(1)) == [5, 4]
    assert list(p.lru_list()) == [3]
    p.append(2, np.ones((8, 1, 1), np.float32), np.ones((8, 1, 1), np.float32))
    # free list (2, 1, 0) then the LRU block 3 is evicted for the 4th block
    assert list(p.block_table(2)) == [2, 1, 0, 3]
    assert not p.is_cached(3) and p.is_cached(5)


# ---- rmsnorm (src/nn/rmsnorm.cpp:4-33), known answers of tests/test_rmsnorm.cpp ----

def test_rmsnorm_known_answers(oracle):
    # tests/test_rmsnorm.cpp:5-14: [3, 4] with unit weight -> [0.8485, 1.1314]
    out = oracle.rmsnorm(np.array([[3.0, 4.0]], np.float32), np.ones(2, np.float32))
    np.testing.assert_allclose(out[0], [0.8485, 1.1314], rtol=1e-3)
    # tests/test_rmsnorm.cpp:16-25: weight [2, 0.5] -> [1.697, 0.5657]
    out = oracle.rmsnorm(np.array([[3.0, 4.0]], np.float32), np.array([2.0, 0.5], np.float32))
    np.testing.assert_allclose(out[0], [1.697, 0.5657], rtol=1e-3)


@needs_ref
@pytest.mark.parametrize("D", [2, 64, 128])
def test_restatement_matches_reference_rmsnorm(oracle, D):
    rng = np.random.default_rng(40 + D)
    x = rng.standard_normal((37, 5, D), dtype=np.float32) * 3
    w = rng.standard_normal(D, dtype=np.float32)
    assert np.array_equal(bits(oracle.rmsnorm(x, w)), bits(oracle.ref_rmsnorm(x, w)))


@pytest.mark.parametrize("name", list(S.FULL_SCENARIOS))
def test_full_scenario_digests_bit_exact(oracle, name):
    """The oracle at BASELINE size (cfg1: 24 layers, prefill 512, 64 decode
    steps): every attention output's SHA-256 equals the reference's, so the
    oracle the GPU tests compare against is pinned bit for bit at full size."""
    g = np.load(os.path.join(GOLDEN, f"{name}_full.npz"))
    res = S.run_scenario(name, OracleBackend())
    outs = S.outputs(res, name)
    keys = [str(k) for k in g["keys"]]
    assert keys == S.output_keys(name)
    bad = [k for k, h in zip(keys, g["sha256"]) if S.digest(outs[k]) != h.tobytes()]
    assert not bad, bad[:5]
    for seq, t in res["tables"].items():
        np.testing.assert_array_equal(t, g[f"table_s{seq}"])
