"""CPU tests of the product library without a GPU: libs1kv.so loads and
exports every entry point include/s1kv.h declares, and the host
bookkeeping (free list, block tables, refcounts, copy-on-write, prefix
cache, LRU) of a host-only pool matches the oracle exactly."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from test_oracle import run_pool_ops  # noqa: F401  (shared op runner)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "s1kv.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(s1kv_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) >= 40, syms


def test_library_exports_every_declared_symbol(s1kv):
    lib = s1kv.lib()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", s1kv.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (s1kv_\w+)", out))
    assert set(declared_symbols()) <= exported


def test_binding_covers_header(s1kv):
    assert set(declared_symbols()) == set(s1kv.SIGNATURES)


def host_pool(s1kv, H, D, max_blocks, bs, layers=1, order=None):
    return s1kv.Pool(layers, H, D, max_blocks, bs, host_only=True, initial_free_list=order)


def test_host_only_pool_refuses_kernels(s1kv):
    p = host_pool(s1kv, 1, 2, 4, 2)
    assert s1kv.lib().s1kv_flush(p.h, None) == s1kv.EINVAL
    b = C.c_void_p()
    seqs = np.zeros(1, np.uint64)
    st = s1kv.lib().s1kv_batch_begin(p.h, seqs.ctypes.data_as(C.POINTER(C.c_uint64)), None, None, 1, None, C.byref(b))
    assert st == s1kv.EINVAL


class ProductOps:
    """Adapter with the oracle Pool's op interface over a host-only pool."""

    def __init__(self, p):
        self.p = p

    def append(self, seq, k, v):
        st, _ = self.p.reserve(seq, k.shape[0])
        return st

    def truncate(self, seq, n):
        try:
            self.p.truncate(seq, n)
            return 0
        except RuntimeError:
            return 1

    def remove(self, seq):
        try:
            self.p.remove(seq)
            return 0
        except RuntimeError:
            return 1

    def length(self, seq):
        return self.p.length(seq)

    def block_table(self, seq):
        return self.p.block_table(seq) if self.p.exists(seq) else None


def test_pool_ops_golden_product(s1kv):
    g = np.load(os.path.join(ROOT, "tests", "golden", "pool_ops.npz"))
    for seed in range(4):
        ops = [tuple(int(x) for x in r) for r in g[f"ops_{seed}"]]
        pr = ProductOps(host_pool(s1kv, 1, 2, 12, 4))
        st, ln, tb = run_pool_ops(pr, ops, seed, lambda p, s, k: p.append(s, k, k))
        np.testing.assert_array_equal(st, g[f"status_{seed}"])
        np.testing.assert_array_equal(ln, g[f"length_{seed}"])
        np.testing.assert_array_equal(tb, g[f"tables_{seed}"])


def test_reserve_partial_progress_on_exhaustion(s1kv, oracle):
    p = host_pool(s1kv, 1, 1, 3, 4)
    o = oracle.Pool(1, 1, 3, 4)
    st, slots = p.reserve(0, 14)   # 12 fit
    rc, oslots, _ = o.reserve(0, 14)
    assert st == s1kv.ENOBLOCKS and rc == oracle.ENOBLOCKS
    np.testing.assert_array_equal(slots, oslots)
    assert p.length(0) == o.length(0) == 12


def test_initial_free_list_permutation_checked(s1kv):
    with pytest.raises(s1kv.S1KVError):
        host_pool(s1kv, 1, 1, 4, 2, order=[0, 1, 1, 2])


def random_sharing_ops(seed, n_ops=400, n_seqs=8):
    rng = np.random.default_rng(seed)
    ops = []
    for _ in range(n_ops):
        r = rng.random()
        a = int(rng.integers(0, n_seqs))
        b = int(rng.integers(0, n_seqs))
        if r < 0.35:
            ops.append(("reserve", a, int(rng.integers(0, 23))))
        elif r < 0.47:
            ops.append(("truncate", a, int(rng.integers(0, 40))))
        elif r < 0.57:
            ops.append(("remove", a, 0))
        elif r < 0.70:
            ops.append(("fork", a, b, int(rng.integers(0, 40))))
        elif r < 0.85:
            ops.append(("insert", a, int(rng.integers(0, 40))))
        else:
            ops.append(("match", b, int(rng.integers(0, 40))))
    return ops


def tokens_for(seq, n):
    """Token ids of a sequence's first n positions: two families of
    sequences share prefixes, so the cache hits."""
    return (np.arange(n, dtype=np.int32) * 7 + (seq % 2)) % 5


@pytest.mark.parametrize("seed", range(12))
def test_sharing_semantics_match_oracle(s1kv, oracle, seed):
    """Random reserve / truncate / remove / fork / prefix insert / prefix
    match scripts: tables, lengths, refcounts, free list and LRU order must
    be identical to the oracle after every op."""
    max_blocks, bs = 24, 4
    order = np.random.default_rng(seed).permutation(max_blocks).astype(np.int32)
    p = host_pool(s1kv, 1, 2, max_blocks, bs, order=order)
    o = oracle.Pool(1, 2, max_blocks, bs, free_order=order)
    for op in random_sharing_ops(seed):
        kind = op[0]
        if kind == "reserve":
            _, a, n = op
            st, slots = p.reserve(a, n)
            rc, oslots, _ = o.reserve(a, n)
            assert (st == 0) == (rc == 0), op
            np.testing.assert_array_equal(slots, oslots)
        elif kind == "truncate":
            _, a, n = op
            ok = o.truncate(a, n) == 0
            if ok:
                p.truncate(a, n)
            else:
                with pytest.raises(RuntimeError):
                    p.truncate(a, n)
        elif kind == "remove":
            _, a, _ = op
            ok = o.remove(a) == 0
            if ok:
                p.remove(a)
            else:
                with pytest.raises(RuntimeError):
                    p.remove(a)
        elif kind == "fork":
            _, a, b, n = op
            rc = o.fork(a, b, n)
            if rc == 0:
                p.fork(a, b, n)
            else:
                with pytest.raises(RuntimeError):
                    p.fork(a, b, n)
        elif kind == "insert":
            _, a, n = op
            if o.has(a) and n <= o.length(a):
                assert p.prefix_insert(a, tokens_for(a, n)) == o.prefix_insert(a, tokens_for(a, n))
        else:
            _, b, n = op
            if not o.has(b):
                rc, hit = o.prefix_match(b, tokens_for(b, n))
                assert p.prefix_match(b, tokens_for(b, n)) == hit
        for s in range(8):
            assert p.exists(s) == o.has(s), (op, s)
            if o.has(s):
                np.testing.assert_array_equal(p.block_table(s), o.block_table(s), err_msg=str(op))
                assert p.length(s) == o.length(s)
        np.testing.assert_array_equal(p.free_list(), o.free_list(), err_msg=str(op))
        np.testing.assert_array_equal(p.lru_list(), o.lru_list(), err_msg=str(op))
        np.testing.assert_array_equal(p.refcounts(), o.refcounts(), err_msg=str(op))


def test_block_hash_matches_oracle(s1kv, oracle):
    t = np.arange(16, dtype=np.int32) * 31
    h1 = s1kv.lib().s1kv_block_hash(0, t.ctypes.data_as(C.POINTER(C.c_int32)), 16)
    assert h1 == oracle.block_hash(0, t)
    h2 = s1kv.lib().s1kv_block_hash(h1, t.ctypes.data_as(C.POINTER(C.c_int32)), 16)
    assert h2 == oracle.block_hash(h1, t) and h2 != h1
