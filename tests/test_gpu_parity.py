"""GPU parity: every kernel of libs1kv against the CPU oracle on the same
seeded inputs, through the C ABI.

Tolerances (stated by the task for this path):
  * appended K/V bytes, block tables, slots: bit-exact;
  * fp32 attention outputs: max |out - ref| <= 2e-5 * max |ref|;
  * bf16-storage attention: <= 1e-2 * max |ref| against the fp32 oracle, and
    <= 2e-5 * max |ref| against the oracle run on the same bf16-rounded K/V.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import scenarios as S  # noqa: E402

pytestmark = pytest.mark.gpu

TOL_F32 = 2e-5
TOL_BF16 = 1e-2


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def host(t):
    return t.detach().cpu().numpy()


@pytest.fixture(autouse=True)
def clean_error_word(s1kv, cuda):
    """Every test starts with a clear device error word, so a flag left by
    one test cannot fail another."""
    try:
        s1kv.device_check(0)
    except s1kv.S1KVError:
        pass
    yield


# ------------------------------------------------------------------ RoPE ---

def test_apply_rope_matches_golden(s1kv, cuda):
    g = np.load(os.path.join(HERE, "golden", "rope.npz"))
    for D in (4, 64, 128):
        for pos in (0, 1, 4095, 131071):
            got = host(s1kv.apply_rope(g[f"x_{D}"], pos))
            assert np.array_equal(bits(got), bits(g[f"out_{D}_{pos}"])), (D, pos)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("D", [64, 128, 6])
def test_rope_append_bit_exact(s1kv, oracle, cuda, dtype, D):
    rng = np.random.default_rng(D)
    Hkv, Hq, n, max_blocks, bs = 2, 6, 300, 40, 16
    order = rng.permutation(max_blocks).astype(np.int32)
    pool = s1kv.Pool(2, Hkv, D, max_blocks, bs, dtype=dtype, initial_free_list=order)
    # three sequences, interleaved reservations, positions up to ~70k
    slots, pos = [], []
    for seq, cnt, start in ((0, 120, 0), (1, 100, 70000), (2, 80, 5)):
        st, sl = pool.reserve(seq, cnt)
        assert st == 0
        slots.append(sl)
        pos.append(np.arange(cnt, dtype=np.int32) + start)
    slots, pos = np.concatenate(slots), np.concatenate(pos)
    k = rng.standard_normal((n, Hkv, D), dtype=np.float32) * 3
    v = rng.standard_normal((n, Hkv, D), dtype=np.float32)
    q = rng.standard_normal((n, Hq, D), dtype=np.float32)
    q_rot = pool.rope_append(1, k, v, slots, pos, q=q)
    cuda.cuda.synchronize()
    k_ref = oracle.apply_rope(k, pos=pos)
    q_ref = oracle.apply_rope(q, pos=pos)
    assert np.array_equal(bits(host(q_rot)), bits(q_ref))
    kst, vst = pool.read_storage(1, s1kv.K), pool.read_storage(1, s1kv.V)
    if dtype == "f32":
        assert np.array_equal(bits(kst[slots]), bits(k_ref))
        assert np.array_equal(bits(vst[slots]), bits(v))
    else:
        assert np.array_equal(kst[slots], oracle.to_bf16_bits(k_ref))
        assert np.array_equal(vst[slots], oracle.to_bf16_bits(v))
    # layer 0 untouched, unwritten slots still zero (zero-filled like the reference)
    assert not pool.read_storage(0, s1kv.K).any()
    mask = np.ones(max_blocks * bs, bool)
    mask[slots] = False
    assert not kst[mask].any()
    assert pool.check_device() == 0


def test_plain_append_and_gather(s1kv, cuda):
    rng = np.random.default_rng(3)
    pool = s1kv.Pool(1, 3, 40, 20, 16, initial_free_list=rng.permutation(20))
    k = rng.standard_normal((77, 3, 40), dtype=np.float32)
    v = rng.standard_normal((77, 3, 40), dtype=np.float32)
    st, slots = pool.reserve(4, 77)
    assert st == 0
    pool.append(0, k, v, slots)
    assert np.array_equal(bits(host(pool.gather(0, 4, s1kv.K))), bits(k))
    assert np.array_equal(bits(host(pool.gather(0, 4, s1kv.V))), bits(v))


# ------------------------------------------------- golden scenarios (GPU) ---

class ProductBackend:
    """Drives a multi-layer device pool with the reference's per-layer call
    order: reservation on layer 0, the same slots reused by later layers."""

    def __init__(self, s1kv, dtype="f32"):
        self.s1kv, self.dtype = s1kv, dtype

    def new_pools(self, layers, H, D, max_blocks, bs, order):
        self.pool = self.s1kv.Pool(layers, H, D, max_blocks, bs, dtype=self.dtype, initial_free_list=order)
        self.layers = layers
        self.lengths = {}
        self.slots = {}

    def rope(self, x, pos):
        return self.s1kv.apply_rope(x, pos)

    def length(self, seq, layer=0):
        return self.lengths.get((seq, layer), 0)

    def append(self, layer, seq, k, v):
        n = k.shape[0]
        if layer == 0:
            st, sl = self.pool.reserve(seq, n)
            assert st == 0
            self.slots[seq] = sl
        self.pool.append(layer, k, v, self.slots[seq])
        self.lengths[(seq, layer)] = self.length(seq, layer) + n

    def attention(self, layer, seq, q, Hq):
        q = q if not hasattr(q, "detach") else q
        out = self.pool.attention(layer, [seq], [q.shape[0]], q, Hq)
        return host(out)

    def table(self, seq):
        return self.pool.block_table(seq)


@pytest.mark.parametrize("name", list(S.SCENARIOS))
def test_scenarios_against_golden(s1kv, cuda, name):
    g = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    got = S.flatten(S.run_scenario(name, ProductBackend(s1kv)), name)
    for key in g.files:
        if key.startswith("table"):
            np.testing.assert_array_equal(got[key], g[key], err_msg=key)
        else:
            assert rel_err(got[key], g[key]) <= TOL_F32, (key, rel_err(got[key], g[key]))


# ------------------------------------------------ batched step vs oracle ---

def build_batch_case(s1kv, oracle, dtype, Hq, Hkv, D, ctx, layers, seed, steps):
    """Prefills `ctx` tokens per sequence through the batch API (layer by
    layer), then runs `steps` fused decode steps (RoPE+append of q/k and
    attention); returns product and oracle outputs per step."""
    import torch
    rng = np.random.default_rng(seed)
    bs = 16
    need = sum((c + steps + bs - 1) // bs for c in ctx)
    max_blocks = int(need * 1.25) + 4
    order = rng.permutation(max_blocks).astype(np.int32)
    pool = s1kv.Pool(layers, Hkv, D, max_blocks, bs, dtype=dtype, initial_free_list=order)
    opools = [oracle.Pool(Hkv, D, max_blocks, bs, free_order=order) for _ in range(layers)]
    seqs = list(range(100, 100 + len(ctx)))
    dev = "cuda"
    # prefill (no attention rows)
    with pool.batch(seqs, ctx, [0] * len(ctx)) as b:
        for layer in range(layers):
            ks, vs = [], []
            for si, c in enumerate(ctx):
                k = rng.standard_normal((c, Hkv, D), dtype=np.float32)
                v = rng.standard_normal((c, Hkv, D), dtype=np.float32)
                kr = oracle.apply_rope(k, 0)
                if dtype == "bf16":
                    kr_o, v_o = oracle.bf16_round(kr), oracle.bf16_round(v)
                else:
                    kr_o, v_o = kr, v
                assert opools[layer].append(seqs[si], kr_o, v_o) == 0
                ks.append(k)
                vs.append(v)
            pos = np.concatenate([np.arange(c, dtype=np.int32) for c in ctx])
            # product: fused RoPE+append of the prefill K (positions from the batch)
            b.rope_append(layer, torch.from_numpy(np.concatenate(ks)).to(dev),
                          torch.from_numpy(np.concatenate(vs)).to(dev))
            del pos
    outs = []
    for step in range(steps):
        with pool.batch(seqs, [1] * len(ctx)) as b:
            step_out = []
            for layer in range(layers):
                q = rng.standard_normal((len(ctx), Hq, D), dtype=np.float32)
                k = rng.standard_normal((len(ctx), Hkv, D), dtype=np.float32)
                v = rng.standard_normal((len(ctx), Hkv, D), dtype=np.float32)
                qt, kt, vt = (torch.from_numpy(x).to(dev) for x in (q, k, v))
                q_rot = b.rope_append(layer, kt, vt, q=qt)
                out = host(b.attention(layer, q_rot))
                ref, ref32 = [], []
                for si, seq in enumerate(seqs):
                    p0 = opools[layer].length(seq)
                    qr = oracle.apply_rope(q[si:si + 1], p0)
                    kr = oracle.apply_rope(k[si:si + 1], p0)
                    if dtype == "bf16":
                        assert opools[layer].append(seq, oracle.bf16_round(kr), oracle.bf16_round(v[si:si + 1])) == 0
                    else:
                        assert opools[layer].append(seq, kr, v[si:si + 1]) == 0
                    ref.append(opools[layer].attention(seq, qr, Hq))
                step_out.append((out, np.concatenate(ref)))
            outs.append(step_out)
    tables_ok = all(np.array_equal(pool.block_table(s), opools[0].block_table(s)) for s in seqs)
    return pool, opools, seqs, outs, tables_ok


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("shape", [(32, 8, 128), (14, 2, 64), (16, 2, 128), (8, 8, 128)])
def test_batched_decode_vs_oracle(s1kv, oracle, cuda, dtype, shape):
    Hq, Hkv, D = shape
    rng = np.random.default_rng(Hq * 7 + D)
    ctx = [int(c) for c in rng.integers(1, 700, size=6)] + [1, 16, 17, 1500]
    pool, opools, seqs, outs, tables_ok = build_batch_case(s1kv, oracle, dtype, Hq, Hkv, D, ctx, 2, 7, 3)
    assert tables_ok
    for step in outs:
        for out, ref in step:
            assert rel_err(out, ref) <= TOL_F32, rel_err(out, ref)
    # appended bytes of the last layer equal the oracle's pool (bit-exact)
    kst = pool.read_storage(1, s1kv.K)
    ok_, _ = opools[1].storage()
    for s in seqs:
        t = pool.block_table(s)
        n = pool.length(s)
        rows = (t[np.arange(n) // 16] * 16 + np.arange(n) % 16)
        if dtype == "f32":
            assert np.array_equal(bits(kst[rows]), bits(ok_[rows]))
        else:
            assert np.array_equal(kst[rows], oracle.to_bf16_bits(ok_[rows]))
    assert pool.check_device() == 0


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_long_rows_capped_splits_vs_oracle(s1kv, oracle, cuda, dtype):
    """Rows long enough for the split planner's cap of 64 splits per row
    (one KV head, 8 query heads; 40,000 tokens = 2,500 tiles -> splits of 40
    tiles, 63 of them): the row merges in two levels -- the last CTA of
    each group of 16 splits merges the group (the last group holds 15), then
    the last group merges the 4 group results (16-byte loads, eight
    partials in flight).  The 10,800-token row takes 17 splits (a group of
    16 and a group of one), the 9,000-token row 15 (one level), the
    300-token row one.  Each row against the oracle's contiguous GQA
    attention, 2e-5 x max |ref| (bf16: on the bf16-rounded K/V)."""
    import torch
    Hq, Hkv, D, bs = 8, 1, 128, 16
    ctx = [40000, 10800, 9000, 300]
    B = len(ctx)
    rng = np.random.default_rng(31)
    k = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    v = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    q = rng.standard_normal((B, Hq, D), dtype=np.float32)
    need = sum((c + bs - 1) // bs for c in ctx)
    pool = s1kv.Pool(1, Hkv, D, need + 4, bs, dtype=dtype,
                     initial_free_list=np.random.default_rng(5).permutation(need + 4))
    seqs = list(range(B))
    with pool.batch(seqs, ctx, [0] * B) as b:
        b.append(0, torch.from_numpy(np.concatenate(k)).cuda(), torch.from_numpy(np.concatenate(v)).cuda())
    with pool.batch(seqs, [0] * B, [1] * B) as b:
        split_tokens, _ = b.plan()
        out = host(b.attention(0, torch.from_numpy(q).cuda()))
    assert split_tokens == 40 * 16
    assert [(c + split_tokens - 1) // split_tokens for c in ctx] == [63, 17, 15, 1]
    for s in range(B):
        kk = oracle.bf16_round(k[s]) if dtype == "bf16" else k[s]
        vv = oracle.bf16_round(v[s]) if dtype == "bf16" else v[s]
        ref = oracle.gqa_attention(q[s:s + 1], kk, vv, Hq, Hkv, D)
        assert rel_err(out[s:s + 1], ref) <= TOL_F32, (s, rel_err(out[s:s + 1], ref))
    assert pool.check_device() == 0
    pool.close()


def test_bf16_storage_within_tolerance(s1kv, oracle, cuda):
    """bf16 K/V storage against the fp32 oracle (no rounding): 1e-2."""
    import torch
    rng = np.random.default_rng(77)
    Hq, Hkv, D, bs = 32, 8, 128, 16
    ctx = [300, 1000, 77]
    pool = s1kv.Pool(1, Hkv, D, 120, bs, dtype="bf16")
    op = oracle.Pool(Hkv, D, 120, bs)
    seqs = [1, 2, 3]
    with pool.batch(seqs, ctx, [0, 0, 0]) as b:
        ks = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
        vs = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
        b.append(0, torch.from_numpy(np.concatenate(ks)).cuda(), torch.from_numpy(np.concatenate(vs)).cuda())
    for s, k, v in zip(seqs, ks, vs):
        op.append(s, k, v)
    q = rng.standard_normal((3, Hq, D), dtype=np.float32)
    out = host(pool.attention(0, seqs, [1, 1, 1], q, Hq))
    ref = np.concatenate([op.attention(s, q[i:i + 1], Hq) for i, s in enumerate(seqs)])
    assert rel_err(out, ref) <= TOL_BF16


# --------------------------------------------------- sharing on the GPU ---

def test_fork_cow_device_bytes(s1kv, oracle, cuda):
    """Fork a 2050-token prefix (128 full blocks + a 2-token tail) to many
    sequences; each append copies the shared tail first (copy-on-write).
    Device bytes, tables and refcounts equal the oracle's."""
    import torch
    rng = np.random.default_rng(2)
    Hkv, D, bs, P = 2, 64, 16, 2050
    max_blocks = 200
    order = rng.permutation(max_blocks).astype(np.int32)
    pool = s1kv.Pool(1, Hkv, D, max_blocks, bs, initial_free_list=order)
    op = oracle.Pool(Hkv, D, max_blocks, bs, free_order=order)
    k = rng.standard_normal((P, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((P, Hkv, D), dtype=np.float32)
    with pool.batch([0], [P], [0]) as b:
        b.append(0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    op.append(0, k, v)
    for dst in range(1, 9):
        pool.fork(0, dst, P)
        op.fork(0, dst, P)
    for dst in range(1, 9):
        n = int(rng.integers(1, 40))
        k2 = rng.standard_normal((n, Hkv, D), dtype=np.float32)
        with pool.batch([dst], [n], [0]) as b:
            b.append(0, torch.from_numpy(k2).cuda(), torch.from_numpy(k2).cuda())
        op.append(dst, k2, k2)
    assert pool.stats()["cow_copies"] == 8
    np.testing.assert_array_equal(pool.refcounts(), op.refcounts())
    kst, vst = pool.read_storage(0, s1kv.K), pool.read_storage(0, s1kv.V)
    ok_, ov = op.storage()
    for s in range(9):
        np.testing.assert_array_equal(pool.block_table(s), op.block_table(s))
        t = pool.block_table(s)
        n = pool.length(s)
        rows = t[np.arange(n) // bs] * bs + np.arange(n) % bs
        assert np.array_equal(bits(kst[rows]), bits(ok_[rows]))
        assert np.array_equal(bits(vst[rows]), bits(ov[rows]))
    q = rng.standard_normal((1, 8, D), dtype=np.float32)
    out = host(pool.attention(0, [5], [1], q, 8))
    assert rel_err(out, op.attention(5, q, 8)) <= TOL_F32


def test_explicit_cow_copy_kernel(s1kv, cuda):
    rng = np.random.default_rng(4)
    pool = s1kv.Pool(3, 2, 64, 10, 16)
    st, slots = pool.reserve(0, 50)
    for layer in range(3):
        k = rng.standard_normal((50, 2, 64), dtype=np.float32)
        pool.append(layer, k, k * 2, slots)
    src = pool.block_table(0)[:2]
    dst = np.array([0, 1], np.int32)
    pool.cow_copy(src, dst)
    for layer in range(3):
        for which in (s1kv.K, s1kv.V):
            st_ = pool.read_storage(layer, which)
            for s_, d_ in zip(src, dst):
                assert np.array_equal(bits(st_[d_ * 16:(d_ + 1) * 16]), bits(st_[s_ * 16:(s_ + 1) * 16]))


# -------------------------------------------- reference interface on GPU ---

def _t(vals):
    return np.asarray(vals, np.float32).reshape(len(vals), 1, 1)


def test_reference_kv_block_pool_cases_on_gpu(s1kv, cuda):
    """tests/test_kv_block_pool.cpp:6-207 through the KVBlockPool mirror."""
    KV = s1kv.KVBlockPool
    p = KV(1, 2, 4, 4)
    k = np.arange(1, 7, dtype=np.float32).reshape(3, 1, 2)
    p.append(0, k, k * 10)
    np.testing.assert_array_equal(host(p.get_k(0)), k)
    np.testing.assert_array_equal(host(p.get_v(0)), k * 10)
    p = KV(1, 1, 4, 2)
    p.append(0, _t([1, 2, 3, 4, 5]), _t([10, 20, 30, 40, 50]))
    np.testing.assert_array_equal(host(p.get_k(0)).ravel(), [1, 2, 3, 4, 5])
    p = KV(1, 1, 4, 4)
    p.append(0, _t([1, 2, 3]), _t([1, 2, 3]))
    p.append(0, _t([4, 5, 6]), _t([4, 5, 6]))
    np.testing.assert_array_equal(host(p.get_k(0)).ravel(), [1, 2, 3, 4, 5, 6])
    p = KV(1, 1, 1, 2)
    p.append(0, _t([1, 2]), _t([1, 2]))
    with pytest.raises(RuntimeError):
        p.append(1, _t([1, 2]), _t([1, 2]))
    p.remove(0)
    p.append(1, _t([1, 2]), _t([1, 2]))
    np.testing.assert_array_equal(host(p.get_k(1)).ravel(), [1, 2])
    with pytest.raises(RuntimeError):
        p.get_k(0)
    p = KV(1, 1, 4, 2)
    with pytest.raises(RuntimeError):
        p.get_k(99)
    assert p.length(0) == 0
    p = KV(1, 1, 4, 4)
    p.append(0, _t(range(1, 11)), _t(range(1, 11)))
    p.truncate(0, 5)
    p.append(0, _t([100, 101]), _t([100, 101]))
    np.testing.assert_array_equal(host(p.get_k(0)).ravel(), [1, 2, 3, 4, 5, 100, 101])
    p = KV(1, 1, 4, 4)
    p.append(0, _t(range(1, 11)), _t(range(1, 11)))
    p.truncate(0, 8)
    p.append(1, _t([1, 2, 3, 4, 5]), _t([1, 2, 3, 4, 5]))
    p = KV(1, 1, 4, 4)
    p.append(0, _t([1, 2, 3, 4]), _t([1, 2, 3, 4]))
    p.truncate(0, 0)
    assert p.length(0) == 0
    p.append(1, _t([9.0] * 16), _t([9.0] * 16))


def test_reference_attention_cases_on_gpu(s1kv, oracle, cuda):
    """tests/test_attention.cpp:29-120 through the mirror (generic kernel)."""
    Q = np.ones((2, 2, 2), np.float32)
    K = np.array([1, 0, 1, 0], np.float32).reshape(2, 1, 2)
    V = np.array([2, 4, 6, 8], np.float32).reshape(2, 1, 2)
    out = host(s1kv.gqa_attention(Q, K, V, 2, 1, 2))
    np.testing.assert_allclose(out[0], [[2, 4], [2, 4]], rtol=1e-6)
    np.testing.assert_allclose(out[1], [[4, 6], [4, 6]], rtol=1e-6)
    p = s1kv.KVBlockPool(1, 2, 4, 2)
    filler = np.zeros((2, 1, 2), np.float32)
    p.append(1, filler, filler)
    p.append(2, filler, filler)
    p.remove(1)
    K = np.array([1, -1, 2, -2, 3, -3, 4, -4, 5, -5], np.float32).reshape(5, 1, 2)
    V = np.array([10, 100, 20, 200, 30, 300, 40, 400, 50, 500], np.float32).reshape(5, 1, 2)
    p.append(0, K, V)
    assert list(p.get_k_view(0).block_table) == [3, 1, 0]
    Q = (np.arange(1, 21, dtype=np.float32) / 10).reshape(5, 2, 2)
    expected = host(s1kv.gqa_attention(Q, p.get_k(0), p.get_v(0), 2, 1, 2))
    actual = host(s1kv.gqa_attention_paged(Q, p.get_k_view(0), p.get_v_view(0), 2, 1, 2))
    assert rel_err(actual, expected) <= TOL_F32
    assert rel_err(actual, oracle.gqa_attention(Q, K, V, 2, 1, 2)) <= TOL_F32


@pytest.mark.parametrize("seed", range(4))
def test_generic_kernel_random_shapes(s1kv, oracle, cuda, seed):
    rng = np.random.default_rng(500 + seed)
    Hkv = int(rng.choice([1, 2, 3]))
    G = int(rng.choice([1, 3, 5]))
    D = int(rng.choice([2, 10, 48, 256]))
    bs = int(rng.choice([1, 4, 8, 32]))
    T = int(rng.integers(1, 200))
    ql = int(rng.integers(1, T + 1))
    k = rng.standard_normal((T, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, D), dtype=np.float32)
    q = rng.standard_normal((ql, G * Hkv, D), dtype=np.float32)
    nb = (T + bs - 1) // bs + 2
    order = rng.permutation(nb)
    p = s1kv.KVBlockPool(Hkv, D, nb, bs, initial_free_list=order)
    op = oracle.Pool(Hkv, D, nb, bs, free_order=order)
    p.append(3, k, v)
    op.append(3, k, v)
    out = host(s1kv.gqa_attention_paged(q, p.get_k_view(3), p.get_v_view(3), G * Hkv, Hkv, D))
    assert rel_err(out, op.attention(3, q, G * Hkv)) <= TOL_F32
    out2 = host(s1kv.gqa_attention(q, k, v, G * Hkv, Hkv, D))
    assert rel_err(out2, oracle.gqa_attention(q, k, v, G * Hkv, Hkv, D)) <= TOL_F32


def test_device_bounds_check_sets_error_word(s1kv, cuda):
    """An out-of-range slot is refused by the append kernel's own bounds
    check (nothing is written) and reported through the error word."""
    pool = s1kv.Pool(1, 1, 16, 2, 16)
    k = np.ones((2, 1, 16), np.float32)
    pool.append(0, k, k, np.array([0, 10_000], np.int32))
    with pytest.raises(s1kv.S1KVError) as e:
        pool.check_device()
    assert e.value.status == s1kv.EDEVICE
    st = pool.read_storage(0, s1kv.K)
    assert st[0].all() and not st[1:].any()
    assert pool.check_device() == 0  # cleared


def test_disk_prefix_round_trip(s1kv, tmp_path, cuda):
    """save_prefix_cache / load_prefix_cache format (src/demo.cpp:10-41)."""
    import torch
    rng = np.random.default_rng(9)
    pool = s1kv.Pool(3, 2, 64, 30, 16)
    k = rng.standard_normal((3, 45, 2, 64), dtype=np.float32)
    v = rng.standard_normal((3, 45, 2, 64), dtype=np.float32)
    with pool.batch([0], [45], [0]) as b:
        for layer in range(3):
            b.append(layer, torch.from_numpy(k[layer]).cuda(), torch.from_numpy(v[layer]).cuda())
    path = tmp_path / "prefix.bin"
    pool.prefix_save(0, path)
    raw = np.fromfile(path, np.float32).reshape(3, 2, 45, 2, 64)
    assert np.array_equal(bits(raw[:, 0]), bits(k)) and np.array_equal(bits(raw[:, 1]), bits(v))
    pool.prefix_load(7, 45, path)
    for layer in range(3):
        assert np.array_equal(bits(host(pool.gather(layer, 7, s1kv.K))), bits(k[layer]))
    with pytest.raises(s1kv.S1KVError):
        pool.prefix_load(8, 46, path)
