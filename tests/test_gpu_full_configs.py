"""GPU parity at the workload sizes of the benchmark configs, through the C
ABI (batch API: s1kv_batch_begin / rope_append / attention), against the CPU
oracle on the same seeded inputs.

  cfg1  exactly as stated: 24 layers, Hq14/Hkv2/D64, RoPE theta 1e6, fp32,
        block 16, shuffled free list, prefill 512 tokens then 64 decode
        steps (seed 0).  The oracle's outputs are pinned bit for bit to the
        reference's by SHA-256 (tests/golden/cfg1_full.npz, made from the
        reference compiled from its sources); every product output within
        2e-5 x max|ref| of the oracle; block table and appended bytes exact.
  cfg2  one layer of the full batch: 64 sequences, contexts U[128, 4096]
        (seed 1), Hq32/Hkv8/D128, pool 1.25x need, permuted; RoPE+append of
        every context token, then two decode steps; fp32 and bf16 storage.
  cfg3  one layer: 256 sequences fork a 2050-token prefix (128 full blocks
        and a shared 2-token tail), each appends a suffix of U[64, 512]
        tokens (copy-on-write of the tail), the prefix-hit prefill over bf16
        K/V, then two decode steps.
  cfg4  the per-GPU shape of the 8-GPU head-sharded run: 4 rows of 131,072
        tokens on one KV head with its 8 query heads, bf16, pool 1.1x need
        scattered (seed 3).

Tolerances: bytes, slots, tables, refcounts bit-exact; fp32 attention (and
bf16-storage decode against the oracle on the same bf16-rounded K/V) within
2e-5 x max|ref|; bf16 storage against the fp32 oracle within 1e-2; the
tensor-core prefill (bf16 Q and P) within PREFILL_TOL of the oracle on the
same rounded K/V, with a median over the 256 sequences within
PREFILL_MEDIAN_TOL.  Measured errors are printed (pytest -s)."""
import concurrent.futures as cf
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
PREFILL_TOL = 1e-2
PREFILL_MEDIAN_TOL = 5e-3
THREADS = min(32, os.cpu_count() or 1)


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def host(t):
    return t.detach().cpu().numpy()


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def pmap(fn, items, workers=THREADS):
    """The oracle's attention calls in parallel host threads (the C calls
    release the GIL; attention only reads the oracle pool)."""
    with cf.ThreadPoolExecutor(workers) as ex:
        return list(ex.map(fn, items))


def storage_rows(pool_len, table, bs=16):
    n = pool_len
    return table[np.arange(n) // bs] * bs + np.arange(n) % bs


@pytest.fixture(autouse=True)
def clean_error_word(s1kv, cuda):
    try:
        s1kv.device_check(0)
    except s1kv.S1KVError:
        pass
    yield


# ------------------------------------------------------------------ cfg1 ---

class OracleBackend:
    def __init__(self, oracle):
        self.O = oracle

    def new_pools(self, layers, H, D, max_blocks, bs, order):
        self.pools = [self.O.Pool(H, D, max_blocks, bs, free_order=order) for _ in range(layers)]

    def rope(self, x, pos):
        return self.O.apply_rope(x, pos)

    def append(self, layer, seq, k, v):
        assert self.pools[layer].append(seq, k, v) == 0

    def attention(self, layer, seq, q, Hq):
        return self.pools[layer].attention(seq, q, Hq)

    def length(self, seq, layer=0):
        return self.pools[layer].length(seq)

    def table(self, seq):
        return self.pools[0].block_table(seq)


def run_cfg1_product(s1kv, name="cfg1"):
    """The scenario through the batch API: one batch for the prefill (512
    appended tokens that are also the 512 query rows), one per decode step;
    per layer the fused RoPE + append (q rotated in the same kernel) and the
    paged attention."""
    sp = S.spec(name)
    order, pre, dec = S.scenario_inputs(name)
    L, seqs = sp["layers"], sp["seqs"]
    pool = s1kv.Pool(L, sp["Hkv"], sp["D"], sp["max_blocks"], sp["bs"], initial_free_list=order)
    outs = {}
    for si, seq in enumerate(seqs):
        with pool.batch([seq], [sp["prefill"][si]]) as b:
            for layer in range(L):
                q, k, v = pre[(layer, seq)]
                q_rot = b.rope_append(layer, dev(k), dev(v), q=dev(q))
                outs[f"prefill_l{layer}_s{seq}"] = host(b.attention(layer, q_rot))
    for step in range(sp["steps"]):
        for seq in seqs:
            with pool.batch([seq], [1]) as b:
                for layer in range(L):
                    q, k, v = dec[(step, seq, layer)]
                    q_rot = b.rope_append(layer, dev(k), dev(v), q=dev(q))
                    outs[f"dec_l{layer}_t{step}_s{seq}"] = host(b.attention(layer, q_rot))
    return pool, outs


def test_cfg1_full_against_pinned_oracle(s1kv, oracle, cuda):
    name = "cfg1"
    g = np.load(os.path.join(HERE, "golden", f"{name}_full.npz"))
    be = OracleBackend(oracle)
    res = S.run_scenario(name, be)
    ref = S.outputs(res, name)
    keys = [str(k) for k in g["keys"]]
    # the oracle at full size is the reference, bit for bit
    assert all(S.digest(ref[k]) == h.tobytes() for k, h in zip(keys, g["sha256"]))
    pool, got = run_cfg1_product(s1kv, name)
    errs = {k: rel_err(got[k], ref[k]) for k in keys}
    worst = max(errs, key=errs.get)
    print(f"cfg1 full: {len(keys)} outputs, worst rel err {errs[worst]:.2e} ({worst})")
    assert errs[worst] <= TOL_F32, (worst, errs[worst])
    for key, prefill in S.kept_values(name):  # directly against the reference's values
        want = g["value/" + key]
        assert rel_err(got[key][-len(want):] if prefill else got[key], want) <= TOL_F32, key
    for seq in S.spec(name)["seqs"]:
        np.testing.assert_array_equal(pool.block_table(seq), g[f"table_s{seq}"])
    # appended K/V bytes of every layer equal the oracle pool's
    t = pool.block_table(0)
    rows = storage_rows(pool.length(0), t)
    for layer in range(S.spec(name)["layers"]):
        ok_, ov = be.pools[layer].storage()
        assert np.array_equal(bits(pool.read_storage(layer, s1kv.K)[rows]), bits(ok_[rows])), layer
        assert np.array_equal(bits(pool.read_storage(layer, s1kv.V)[rows]), bits(ov[rows])), layer
    assert pool.check_device() == 0
    pool.close()


# ------------------------------------------------------------------ cfg2 ---

def cfg2_inputs():
    """The bench's per-GPU batch: 64 contexts U[128, 4096] from seed 1, then
    the pool's permutation and N(0,1) K/V from the same generator."""
    rng = np.random.default_rng(1)
    ctx = [int(c) for c in rng.integers(128, 4097, size=64)]
    steps = 2
    need = sum((c + steps + 15) // 16 for c in ctx)
    max_blocks = int(need * 1.25)
    order = rng.permutation(max_blocks).astype(np.int32)
    T = sum(ctx)
    k = rng.standard_normal((T, 8, 128), dtype=np.float32)
    v = rng.standard_normal((T, 8, 128), dtype=np.float32)
    dec = [tuple(rng.standard_normal((64, h, 128), dtype=np.float32) for h in (32, 8, 8)) for _ in range(steps)]
    return ctx, max_blocks, order, k, v, dec


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_cfg2_full_batch_one_layer(s1kv, oracle, cuda, dtype):
    Hq, Hkv, D = 32, 8, 128
    ctx, max_blocks, order, k, v, dec = cfg2_inputs()
    seqs = list(range(64))
    pool = s1kv.Pool(1, Hkv, D, max_blocks, 16, dtype=dtype, initial_free_list=order, max_seqs=256)
    with pool.batch(seqs, ctx, [0] * 64) as b:
        b.rope_append(0, dev(k), dev(v))
    rnd = oracle.bf16_round if dtype == "bf16" else (lambda a: a)
    op = oracle.Pool(Hkv, D, max_blocks, 16, free_order=order)  # same rounding as the product's storage
    op32 = oracle.Pool(Hkv, D, max_blocks, 16, free_order=order) if dtype == "bf16" else op
    off = 0
    for s, c in zip(seqs, ctx):
        kr = oracle.apply_rope(k[off:off + c], 0)
        assert op.append(s, rnd(kr), rnd(v[off:off + c])) == 0
        if op32 is not op:
            assert op32.append(s, kr, v[off:off + c]) == 0
        off += c
    del k, v
    worst = worst32 = 0.0
    for q, k1, v1 in dec:
        with pool.batch(seqs, [1] * 64) as b:
            q_rot = b.rope_append(0, dev(k1), dev(v1), q=dev(q))
            out = host(b.attention(0, q_rot))
        qr = []
        for i, s in enumerate(seqs):
            p0 = op.length(s)
            qr.append(oracle.apply_rope(q[i:i + 1], p0))
            kr = oracle.apply_rope(k1[i:i + 1], p0)
            assert op.append(s, rnd(kr), rnd(v1[i:i + 1])) == 0
            if op32 is not op:
                assert op32.append(s, kr, v1[i:i + 1]) == 0
        assert np.array_equal(bits(host(q_rot)), bits(np.concatenate(qr)))
        ref = np.concatenate(pmap(lambda i: op.attention(seqs[i], qr[i], Hq), range(64)))
        worst = max(worst, rel_err(out, ref))
        if op32 is not op:
            ref32 = np.concatenate(pmap(lambda i: op32.attention(seqs[i], qr[i], Hq), range(64)))
            worst32 = max(worst32, rel_err(out, ref32))
    print(f"cfg2 {dtype}: 64 seqs, rel err {worst:.2e} vs oracle on the stored values"
          + (f", {worst32:.2e} vs the fp32 oracle" if op32 is not op else ""))
    assert worst <= TOL_F32, worst
    assert worst32 <= TOL_BF16, worst32
    kst, vst = pool.read_storage(0, s1kv.K), pool.read_storage(0, s1kv.V)
    ok_, ov = op.storage()
    for s in seqs:
        t = pool.block_table(s)
        np.testing.assert_array_equal(t, op.block_table(s))
        rows = storage_rows(pool.length(s), t)
        if dtype == "f32":
            assert np.array_equal(bits(kst[rows]), bits(ok_[rows])) and np.array_equal(bits(vst[rows]), bits(ov[rows]))
        else:
            assert np.array_equal(kst[rows], oracle.to_bf16_bits(ok_[rows]))
            assert np.array_equal(vst[rows], oracle.to_bf16_bits(ov[rows]))
    assert pool.check_device() == 0
    pool.close()


# ------------------------------------------------------------------ cfg3 ---

def np_causal_gqa(q, k, v, Hq, Hkv):
    """GQA_attention's arithmetic (src/nn/attention.cpp:13-126: kv head h /
    (Hq/Hkv), scores q.k / sqrt(D), row i of q_len sees keys 0 ..
    (kv_len - q_len) + i, softmax, PV) as float64 BLAS products, for
    checking many long prefill chunks quickly; pinned to the C oracle on a
    sample of the same chunks."""
    Lq, S_, D = q.shape[0], k.shape[0], q.shape[2]
    G = Hq // Hkv
    qg = q.astype(np.float64).reshape(Lq, Hkv, G, D).transpose(1, 0, 2, 3).reshape(Hkv, Lq * G, D)
    kt = k.astype(np.float64).transpose(1, 2, 0)          # [Hkv, D, S]
    sc = (qg @ kt) / np.sqrt(D)                            # [Hkv, Lq*G, S]
    row = np.repeat(np.arange(Lq), G)
    mask = np.arange(S_)[None, :] > (S_ - Lq + row)[:, None]
    sc[:, mask] = -np.inf
    sc -= sc.max(axis=-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(axis=-1, keepdims=True)
    o = p @ v.astype(np.float64).transpose(1, 0, 2)        # [Hkv, Lq*G, D]
    return o.reshape(Hkv, Lq, G, D).transpose(1, 0, 2, 3).reshape(Lq, Hq, D)


def test_cfg3_full_256_forks_prefill_and_decode(s1kv, oracle, cuda):
    Hq, Hkv, D, bs, P, n, dec_steps = 32, 8, 128, 16, 2050, 256, 2
    rng = np.random.default_rng(2)
    suff = [int(x) for x in rng.integers(64, 513, size=n)]
    blocks = (P + bs - 1) // bs + sum((L + dec_steps + bs) // bs + 1 for L in suff) + 8
    order = rng.permutation(blocks).astype(np.int32)
    pool = s1kv.Pool(1, Hkv, D, blocks, bs, dtype="bf16", initial_free_list=order, max_seqs=n + 8)
    op = oracle.Pool(Hkv, D, blocks, bs, free_order=order)
    kp = rng.standard_normal((P, Hkv, D), dtype=np.float32)
    vp = rng.standard_normal((P, Hkv, D), dtype=np.float32)
    with pool.batch([0], [P], [0]) as b:
        b.rope_append(0, dev(kp), dev(vp))
    assert op.append(0, oracle.bf16_round(oracle.apply_rope(kp, 0)), oracle.bf16_round(vp)) == 0
    seqs = list(range(1, n + 1))
    for s in seqs:
        pool.fork(0, s, P)
        assert op.fork(0, s, P) == 0
    T = sum(suff)
    q = rng.standard_normal((T, Hq, D), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, D), dtype=np.float32)
    with pool.batch(seqs, suff) as b:  # copy-on-write of every tail, RoPE + append, prefill
        q_rot = host(b.rope_append(0, dev(k), dev(v), q=dev(q)))
        out = host(b.attention(0, dev(q_rot)))
    starts = np.concatenate([[0], np.cumsum(suff)])
    qr = []
    for i, s in enumerate(seqs):
        a, e = starts[i], starts[i + 1]
        assert op.append(s, oracle.bf16_round(oracle.apply_rope(k[a:e], P)), oracle.bf16_round(v[a:e])) == 0
        qr.append(oracle.apply_rope(q[a:e], P))
    del k, v, q
    assert np.array_equal(bits(q_rot), bits(np.concatenate(qr)))
    assert pool.stats()["cow_copies"] == n
    np.testing.assert_array_equal(pool.refcounts(), op.refcounts())
    kst, vst = pool.read_storage(0, s1kv.K), pool.read_storage(0, s1kv.V)
    ok_, ov = op.storage()
    for s in [0] + seqs:
        t = pool.block_table(s)
        np.testing.assert_array_equal(t, op.block_table(s))
        rows = storage_rows(pool.length(s), t)
        assert np.array_equal(kst[rows], oracle.to_bf16_bits(ok_[rows])), s
        assert np.array_equal(vst[rows], oracle.to_bf16_bits(ov[rows])), s
    del kst, vst

    def np_ref(i):
        s = seqs[i]
        t = op.block_table(s)
        rows = storage_rows(op.length(s), t)
        return np_causal_gqa(qr[i], ok_[rows], ov[rows], Hq, Hkv)

    refs = pmap(np_ref, range(n), workers=4)  # each product is itself multithreaded
    errs = [rel_err(out[starts[i]:starts[i + 1]], refs[i]) for i in range(n)]
    # the float64 restatement agrees with the C oracle on a sample
    sample = list(range(0, n, 16))
    oref = pmap(lambda i: op.attention(seqs[i], qr[i], Hq), sample)
    for i, o in zip(sample, oref):
        assert rel_err(o, refs[i]) <= 1e-5, i
    print(f"cfg3 prefill: 256 seqs x suffix U[64,512] over 2050 + suffix keys, bf16 K/V; rel err vs oracle "
          f"max {max(errs):.2e}, median {np.median(errs):.2e}")
    assert max(errs) <= PREFILL_TOL, max(errs)
    # the bf16 narrowing of Q and P gives 3-7e-3 per sequence (median 3.3e-3
    # measured); a median far above that is a regression, not rounding
    assert np.median(errs) <= PREFILL_MEDIAN_TOL, np.median(errs)
    # two decode steps over the shared prefix blocks
    worst = 0.0
    for _ in range(dec_steps):
        q1 = rng.standard_normal((n, Hq, D), dtype=np.float32)
        k1 = rng.standard_normal((n, Hkv, D), dtype=np.float32)
        v1 = rng.standard_normal((n, Hkv, D), dtype=np.float32)
        with pool.batch(seqs, [1] * n) as b:
            qd = b.rope_append(0, dev(k1), dev(v1), q=dev(q1))
            od = host(b.attention(0, qd))
        qdr = []
        for i, s in enumerate(seqs):
            p0 = op.length(s)
            qdr.append(oracle.apply_rope(q1[i:i + 1], p0))
            kr = oracle.apply_rope(k1[i:i + 1], p0)
            assert op.append(s, oracle.bf16_round(kr), oracle.bf16_round(v1[i:i + 1])) == 0
        ref = np.concatenate(pmap(lambda i: op.attention(seqs[i], qdr[i], Hq), range(n)))
        worst = max(worst, rel_err(od, ref))
    print(f"cfg3 decode after the prefill: rel err {worst:.2e}")
    assert worst <= TOL_F32, worst
    for s in seqs:
        np.testing.assert_array_equal(pool.block_table(s), op.block_table(s))
    assert pool.check_device() == 0
    pool.close()


# ------------------------------------------------------------------ cfg4 ---

def test_cfg4_rank_shape_131072_token_rows(s1kv, oracle, cuda):
    """One rank's share of the 8-GPU KV-head-sharded run: 4 sequences of
    131,072 tokens on one KV head with its 8 query heads, bf16 K/V, blocks
    scattered over a pool of 1.1x need (seed 3), one decode step through the
    batch API (the planner's longest rows: the split merge is exercised)."""
    Hq, Hkv, D, bs, B, CTX = 8, 1, 128, 16, 4, 131072
    need = B * ((CTX + 1 + bs - 1) // bs)
    max_blocks = int(need * 1.1)
    order = np.random.default_rng(3).permutation(max_blocks).astype(np.int32)
    pool = s1kv.Pool(1, Hkv, D, max_blocks, bs, dtype="bf16", initial_free_list=order, max_seqs=8)
    rng = np.random.default_rng(3)
    seqs = list(range(B))
    k = rng.standard_normal((B * CTX, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((B * CTX, Hkv, D), dtype=np.float32)
    with pool.batch(seqs, [CTX] * B, [0] * B) as b:
        b.append(0, dev(k), dev(v))
    kb, vb = oracle.bf16_round(k), oracle.bf16_round(v)
    q = rng.standard_normal((B, Hq, D), dtype=np.float32)
    k1 = rng.standard_normal((B, Hkv, D), dtype=np.float32)
    v1 = rng.standard_normal((B, Hkv, D), dtype=np.float32)
    with pool.batch(seqs, [1] * B) as b:
        split_tokens, n_items = b.plan()
        qr = host(b.rope_append(0, dev(k1), dev(v1), q=dev(q)))
        out = host(b.attention(0, dev(qr)))
    kr1 = oracle.bf16_round(oracle.apply_rope(k1, pos=np.full(B, CTX, np.int32)))
    v1b = oracle.bf16_round(v1)

    def ref(i):
        kk = np.concatenate([kb[i * CTX:(i + 1) * CTX], kr1[i:i + 1]])
        vv = np.concatenate([vb[i * CTX:(i + 1) * CTX], v1b[i:i + 1]])
        return oracle.gqa_attention(qr[i:i + 1], kk, vv, Hq, Hkv, D), np_causal_gqa(qr[i:i + 1], kk, vv, Hq, Hkv)

    refs = pmap(ref, range(B), workers=2)
    # Over 131,073 keys the oracle's own fp32 sums (the reference's
    # sequential loops) are off the exact result by ~1.5-2e-5 of the output
    # scale, so the kernel is held to 2e-5 against the float64 evaluation of
    # the same arithmetic, and to 2e-5 plus the oracle's own error against
    # the oracle.
    err64 = [rel_err(out[i:i + 1], refs[i][1]) for i in range(B)]
    err_or = [rel_err(out[i:i + 1], refs[i][0]) for i in range(B)]
    or64 = [rel_err(refs[i][0], refs[i][1]) for i in range(B)]
    splits = (CTX + 1 + split_tokens - 1) // split_tokens
    print(f"cfg4 rank shape: 4 x 131073 tokens, {splits} splits of {split_tokens} tokens per row, "
          f"{n_items} work items; rel err vs float64 {max(err64):.2e}, vs the oracle {max(err_or):.2e} "
          f"(the oracle vs float64: {max(or64):.2e})")
    assert max(err64) <= TOL_F32, err64
    assert all(e <= TOL_F32 + o for e, o in zip(err_or, or64)), (err_or, or64)
    for s in seqs:
        assert pool.length(s) == CTX + 1
    assert pool.check_device() == 0
    pool.close()


# ----------------------------------------- KV-head sharding on one GPU ---

@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_head_sharded_exchange_on_one_gpu(s1kv, oracle, cuda, dtype):
    """Two ranks of a KV-head-sharded decode emulated in one process on one
    GPU: each rank's pool holds half of the KV heads, its exchange is opened
    on the other's device memory (s1kv_exchange_open_local), and
    s1kv_batch_attention_exchange stores every finished row into both
    ranks' token-major buffers and signals the epoch.  The two ranks' calls
    run one after the other on one stream, so each rank's bounded wait finds
    both flags already set (no kernel waits on a kernel running beside it).
    Three layers alternate the two slots; every gathered output equals the
    oracle's full-head attention, on both ranks."""
    torch = cuda
    Hq, Hkv, D, bs, world = 32, 8, 128, 16, 2
    rng = np.random.default_rng(17)
    ctx = [5000, 130, 2049, 17, 777, 1]
    B, layers = len(ctx), 3
    seqs = list(range(B))
    need = sum((c + 1 + bs - 1) // bs for c in ctx) + 4
    order = rng.permutation(need).astype(np.int32)
    pools = [s1kv.Pool(layers, Hkv // world, D, need, bs, dtype=dtype, initial_free_list=order) for _ in range(world)]
    ops = [oracle.Pool(Hkv, D, need, bs, free_order=order) for _ in range(layers)]
    rnd = oracle.bf16_round if dtype == "bf16" else (lambda a: a)
    T = sum(ctx)
    with pools[0].batch(seqs, ctx, [0] * B) as b0, pools[1].batch(seqs, ctx, [0] * B) as b1:
        for layer in range(layers):
            k = rng.standard_normal((T, Hkv, D), dtype=np.float32)
            v = rng.standard_normal((T, Hkv, D), dtype=np.float32)
            half = Hkv // world
            b0.append(layer, dev(k[:, :half]), dev(v[:, :half]))
            b1.append(layer, dev(k[:, half:]), dev(v[:, half:]))
            off = 0
            for s, c in zip(seqs, ctx):
                assert ops[layer].append(s, rnd(k[off:off + c]), rnd(v[off:off + c])) == 0
                off += c
    exs = [s1kv.PeerExchange(r, world, B, Hq, D, local=True) for r in range(world)]
    s1kv.PeerExchange.open_local(exs)
    hq = Hq // world
    worst = 0.0
    with pools[0].batch(seqs, [0] * B, [1] * B) as b0, pools[1].batch(seqs, [0] * B, [1] * B) as b1:
        for layer in range(layers):
            epoch = layer + 1
            q = rng.standard_normal((B, Hq, D), dtype=np.float32)
            for r, b in enumerate((b0, b1)):
                exs[r].attention(b, layer, dev(q[:, r * hq:(r + 1) * hq]), r * hq, epoch)
            for r in range(world):
                exs[r].wait(epoch, force=True)
            got = [host(exs[r].output(epoch)) for r in range(world)]
            ref = np.concatenate(pmap(lambda i: ops[layer].attention(seqs[i], q[i:i + 1], Hq), range(B)))
            for r in range(world):
                worst = max(worst, rel_err(got[r], ref))
            # the wait fused with a copy of one head range (the other rank's
            # heads, as the next layer's queries): the same bits as the buffer
            for r in range(world):
                h0 = (1 - r) * hq
                dst = torch.full((B, hq, D), float("nan"), device="cuda")
                exs[r].wait_copy(epoch, h0, hq, dst)
                np.testing.assert_array_equal(host(dst), got[r][:, h0:h0 + hq])
    print(f"head-sharded exchange on one GPU ({dtype}): rel err {worst:.2e}")
    assert worst <= TOL_F32, worst
    torch.cuda.synchronize()
    for p in pools:
        assert p.check_device() == 0
    for e in exs:
        e.close()
    for p in pools:
        p.close()
