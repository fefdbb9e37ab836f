"""ctypes loader for the CPU oracle.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only to compare the library's results with it.  It
exposes

  * ``Oracle``     -- the plain-C restatement (oracle/kvoracle.c), built by
                      oracle/Makefile from files in this repository;
  * ``RefOracle``  -- the reference's own CPU code (oracle/_ref/libs1ref.so),
                      present only where the reference sources were compiled.

Both speak numpy arrays.  The reference functions they restate or wrap are
cited in kvoracle.c and ref_capi.cpp.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libs1ref.so")
ROPE_BASE = 1.0e6  # src/nn/RoPE.cpp:22

OK, ENOBLOCKS, ENOSEQ, EINVAL = 0, 1, 2, 3

_lock = threading.Lock()
_lib = None
_ref = None

i64, u64, i32, f32 = C.c_int64, C.c_uint64, C.c_int32, C.c_float
vp = C.c_void_p


def _fp(a):
    return a.ctypes.data_as(vp)


def build():
    """Compile liboracle.so (and _ref when the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _load():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(os.path.join(HERE, "kvoracle.c")):
                build()
            lib = C.CDLL(LIB)
            sig = {
                "kvo_f32_to_bf16": (C.c_uint16, [f32]),
                "kvo_bf16_to_f32": (f32, [C.c_uint16]),
                "kvo_bf16_round_array": (None, [vp, vp, i64]),
                "kvo_to_bf16_array": (None, [vp, vp, i64]),
                "kvo_apply_rope": (None, [vp, i64, i64, i64, i64, f32, vp]),
                "kvo_apply_rope_pos": (None, [vp, i64, i64, i64, vp, f32, vp]),
                "kvo_rope_cs": (None, [i64, i64, i64, f32, vp, vp]),
                "kvo_rmsnorm": (None, [vp, i64, i64, vp, f32, vp]),
                "kvo_gqa_attention": (None, [vp, vp, vp, i64, i64, i64, i64, i64, vp]),
                "kvo_gqa_attention_paged": (None, [vp, i64, vp, vp, vp, i64, i64, i64, i64, i64, vp]),
                "kvo_pool_new": (vp, [i64, i64, i64, i64]),
                "kvo_pool_free": (None, [vp]),
                "kvo_set_free_list": (C.c_int, [vp, vp, i64]),
                "kvo_pool_k": (C.POINTER(f32), [vp]),
                "kvo_pool_v": (C.POINTER(f32), [vp]),
                "kvo_num_free": (i64, [vp]),
                "kvo_num_lru": (i64, [vp]),
                "kvo_free_list": (i64, [vp, vp, i64]),
                "kvo_lru_list": (i64, [vp, vp, i64]),
                "kvo_length": (i64, [vp, u64]),
                "kvo_has_seq": (C.c_int, [vp, u64]),
                "kvo_reserve": (C.c_int, [vp, u64, i64, vp, C.POINTER(i64), C.POINTER(i32), C.POINTER(i32)]),
                "kvo_append": (C.c_int, [vp, u64, vp, vp, i64]),
                "kvo_get": (C.c_int, [vp, u64, C.c_int, vp]),
                "kvo_remove": (C.c_int, [vp, u64]),
                "kvo_truncate": (C.c_int, [vp, u64, i64]),
                "kvo_block_table": (C.c_int, [vp, u64, vp, i64, C.POINTER(i64)]),
                "kvo_refcount": (i32, [vp, i32]),
                "kvo_is_cached": (C.c_int, [vp, i32]),
                "kvo_fork": (C.c_int, [vp, u64, u64, i64]),
                "kvo_block_hash": (u64, [u64, vp, i64]),
                "kvo_prefix_insert": (i64, [vp, u64, vp, i64]),
                "kvo_prefix_match": (C.c_int, [vp, u64, vp, i64, C.POINTER(i64)]),
                "kvo_quantize_rows": (None, [vp, i64, i64, vp, vp]),
                "kvo_matmul_int8": (None, [vp, i64, i64, vp, vp, i64, vp]),
            }
            for name, (res, args) in sig.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def ref_available():
    return os.path.exists(REF_LIB)


def _load_ref():
    global _ref
    with _lock:
        if _ref is None:
            if not ref_available():
                raise FileNotFoundError(REF_LIB)
            lib = C.CDLL(REF_LIB)
            sig = {
                "ref_pool_new": (vp, [i64, i64, i64, i64]),
                "ref_pool_free": (None, [vp]),
                "ref_append": (C.c_int, [vp, u64, vp, vp, i64, i64, i64]),
                "ref_length": (i64, [vp, u64]),
                "ref_remove": (C.c_int, [vp, u64]),
                "ref_truncate": (C.c_int, [vp, u64, i64]),
                "ref_get": (C.c_int, [vp, u64, C.c_int, vp]),
                "ref_block_table": (C.c_int, [vp, u64, vp, i64, C.POINTER(i64)]),
                "ref_pool_base": (C.POINTER(f32), [vp, u64, C.c_int]),
                "ref_apply_rope": (None, [vp, i64, i64, i64, i64, vp]),
                "ref_rmsnorm": (None, [vp, i64, i64, vp, f32, vp]),
                "ref_gqa_attention": (None, [vp, vp, vp, i64, i64, i64, i64, i64, vp]),
                "ref_gqa_attention_paged": (C.c_int, [vp, u64, vp, i64, i64, i64, i64, vp]),
                "ref_decode_batch": (None, [vp, i64, vp, i64, vp, i64, i64, i64, i64, vp]),
                "ref_quantize_tensor": (None, [vp, i64, i64, vp, vp]),
                "ref_matmul_quantized_blocked": (None, [vp, i64, i64, vp, vp, i64, vp]),
                "ref_qt_new": (vp, [vp, vp, i64, i64]),
                "ref_qt_free": (None, [vp]),
                "ref_matmul_quantized": (None, [vp, i64, i64, vp, vp]),
            }
            for name, (res, args) in sig.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _ref = lib
    return _ref


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _vp(a):
    return a.ctypes.data_as(vp)


# ---------------------------------------------------- int8 projections --

def quantize_rows(w):
    """quantize_tensor (src/quantized_tensor.cpp:9-47), restated:
    (q int8 [rows, cols], scales fp32 [rows])."""
    w = _f32(w)
    rows, cols = w.shape
    q = np.empty((rows, cols), np.int8)
    sc = np.empty(rows, np.float32)
    _load().kvo_quantize_rows(_vp(w), rows, cols, _vp(q), _vp(sc))
    return q, sc


def matmul_int8(x, q, scales):
    """matmul_quantized_range_blocked (src/quantized_tensor.cpp:60-100),
    restated: x [M, K] * (q [K, N] scaled per row) -> [M, N], k in order."""
    x = _f32(x)
    q = np.ascontiguousarray(q, dtype=np.int8)
    scales = _f32(scales)
    M, K = x.shape
    N = q.shape[1]
    out = np.empty((M, N), np.float32)
    _load().kvo_matmul_int8(_vp(x), M, K, _vp(q), _vp(scales), N, _vp(out))
    return out


def ref_quantize_rows(w):
    """The reference's quantize_tensor itself (oracle/_ref)."""
    w = _f32(w)
    rows, cols = w.shape
    q = np.empty((rows, cols), np.int8)
    sc = np.empty(rows, np.float32)
    _load_ref().ref_quantize_tensor(_vp(w), rows, cols, _vp(q), _vp(sc))
    return q, sc


def ref_matmul_int8(x, q, scales, threaded=False):
    """The reference's matmul_quantized_range_blocked (one thread) or, with
    `threaded`, matmul_quantized over its ThreadPool (oracle/_ref)."""
    x = _f32(x)
    q = np.ascontiguousarray(q, dtype=np.int8)
    scales = _f32(scales)
    M, K = x.shape
    N = q.shape[1]
    out = np.empty((M, N), np.float32)
    R = _load_ref()
    if threaded:
        qt = R.ref_qt_new(_vp(q), _vp(scales), K, N)
        try:
            R.ref_matmul_quantized(_vp(x), M, K, qt, _vp(out))
        finally:
            R.ref_qt_free(qt)
    else:
        R.ref_matmul_quantized_blocked(_vp(x), M, K, _vp(q), _vp(scales), N, _vp(out))
    return out


# ---------------------------------------------------------------- math ----

def apply_rope(x, start_pos=0, pos=None, base=ROPE_BASE):
    """apply_rope on [T, H, D] (or [T, D]); src/nn/RoPE.cpp:6-39."""
    lib = _load()
    x = _f32(x)
    x3 = x.reshape(x.shape[0], -1, x.shape[-1])
    T, H, D = x3.shape
    out = np.empty_like(x3)
    if pos is None:
        lib.kvo_apply_rope(_fp(x3), T, H, D, start_pos, base, _fp(out))
    else:
        p = np.ascontiguousarray(pos, dtype=np.int32)
        lib.kvo_apply_rope_pos(_fp(x3), T, H, D, _fp(p), base, _fp(out))
    return out.reshape(x.shape)


def rope_table(max_pos, D, base=ROPE_BASE):
    """[max_pos, D/2, 2] cos/sin exactly as the rotation computes them."""
    lib = _load()
    out = np.empty((max_pos, D // 2, 2), np.float32)
    c, s = f32(), f32()
    for p in range(max_pos):
        for j in range(D // 2):
            lib.kvo_rope_cs(p, j, D, base, C.byref(c), C.byref(s))
            out[p, j, 0] = c.value
            out[p, j, 1] = s.value
    return out


def rmsnorm(x, w, eps=1e-6):
    """rmsnorm over the last dim; src/nn/rmsnorm.cpp:4-33."""
    lib = _load()
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    lib.kvo_rmsnorm(_fp(x), x.size // x.shape[-1], x.shape[-1], _fp(w), eps, _fp(out))
    return out


def gqa_attention(q, k, v, Hq, Hkv, D):
    """GQA_attention on contiguous K/V; src/nn/attention.cpp:13-126."""
    lib = _load()
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty((q.shape[0], Hq, D), np.float32)
    lib.kvo_gqa_attention(_fp(q), _fp(k), _fp(v), q.shape[0], k.shape[0], Hq, Hkv, D, _fp(out))
    return out


def gqa_attention_paged(q, pool_k, pool_v, table, kv_len, bs, Hq, Hkv, D):
    """GQA_attention_paged through a block table; src/nn/attention.cpp:128-239."""
    lib = _load()
    q, pool_k, pool_v = _f32(q), _f32(pool_k), _f32(pool_v)
    t = np.ascontiguousarray(table, dtype=np.int32)
    out = np.empty((q.shape[0], Hq, D), np.float32)
    lib.kvo_gqa_attention_paged(_fp(q), q.shape[0], _fp(pool_k), _fp(pool_v), _fp(t), kv_len, bs, Hq, Hkv, D,
                                _fp(out))
    return out


def bf16_round(a):
    """Narrow to bfloat16 (round to nearest even) and widen back to fp32."""
    lib = _load()
    a = _f32(a)
    out = np.empty_like(a)
    lib.kvo_bf16_round_array(_fp(a), _fp(out), a.size)
    return out


def to_bf16_bits(a):
    lib = _load()
    a = _f32(a)
    out = np.empty(a.shape, np.uint16)
    lib.kvo_to_bf16_array(_fp(a), _fp(out), a.size)
    return out


def block_hash(parent, tokens):
    lib = _load()
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    return int(lib.kvo_block_hash(parent, _fp(t), t.size))


# ---------------------------------------------------------------- pool ----

class Pool:
    """One layer's KVBlockPool (src/infer/kv_block_pool.cpp) plus the
    sharing semantics (refcount, fork, copy-on-write, prefix cache + LRU)."""

    def __init__(self, num_heads, head_dim, max_blocks, block_size=16, free_order=None):
        self.lib = _load()
        self.H, self.D, self.max_blocks, self.bs = num_heads, head_dim, max_blocks, block_size
        self.p = self.lib.kvo_pool_new(num_heads, head_dim, max_blocks, block_size)
        if free_order is not None:
            fo = np.ascontiguousarray(free_order, dtype=np.int32)
            assert self.lib.kvo_set_free_list(self.p, _fp(fo), fo.size) == OK

    def __del__(self):
        if getattr(self, "p", None):
            self.lib.kvo_pool_free(self.p)
            self.p = None

    def reserve(self, seq, n):
        slots = np.zeros(max(n, 1), np.int32)
        done, cs, cd = i64(), i32(), i32()
        rc = self.lib.kvo_reserve(self.p, seq, n, _fp(slots), C.byref(done), C.byref(cs), C.byref(cd))
        return rc, slots[: done.value].copy(), (cs.value, cd.value)

    def append(self, seq, k, v):
        k, v = _f32(k), _f32(v)
        return self.lib.kvo_append(self.p, seq, _fp(k), _fp(v), k.shape[0])

    def length(self, seq):
        return int(self.lib.kvo_length(self.p, seq))

    def has(self, seq):
        return bool(self.lib.kvo_has_seq(self.p, seq))

    def get(self, seq, which):
        out = np.empty((self.length(seq), self.H, self.D), np.float32)
        rc = self.lib.kvo_get(self.p, seq, which, _fp(out))
        if rc != OK:
            raise RuntimeError("KVBlockPool: Sequence ID not found")
        return out

    def get_k(self, seq):
        return self.get(seq, 0)

    def get_v(self, seq):
        return self.get(seq, 1)

    def remove(self, seq):
        return self.lib.kvo_remove(self.p, seq)

    def truncate(self, seq, keep):
        return self.lib.kvo_truncate(self.p, seq, keep)

    def block_table(self, seq):
        cap = self.max_blocks + 1
        out = np.zeros(cap, np.int32)
        n = i64()
        rc = self.lib.kvo_block_table(self.p, seq, _fp(out), cap, C.byref(n))
        if rc != OK:
            return None
        return out[: n.value].copy()

    def free_list(self):
        out = np.zeros(self.max_blocks + 1, np.int32)
        n = self.lib.kvo_free_list(self.p, _fp(out), self.max_blocks + 1)
        return out[:n].copy()

    def lru_list(self):
        out = np.zeros(self.max_blocks + 1, np.int32)
        n = self.lib.kvo_lru_list(self.p, _fp(out), self.max_blocks + 1)
        return out[:n].copy()

    def num_free(self):
        return int(self.lib.kvo_num_free(self.p))

    def refcount(self, block):
        return int(self.lib.kvo_refcount(self.p, block))

    def refcounts(self):
        return np.array([self.refcount(b) for b in range(self.max_blocks)], np.int32)

    def is_cached(self, block):
        return bool(self.lib.kvo_is_cached(self.p, block))

    def fork(self, src, dst, n):
        return self.lib.kvo_fork(self.p, src, dst, n)

    def prefix_insert(self, seq, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        return int(self.lib.kvo_prefix_insert(self.p, seq, _fp(t), t.size))

    def prefix_match(self, dst, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        n = i64()
        rc = self.lib.kvo_prefix_match(self.p, dst, _fp(t), t.size, C.byref(n))
        return rc, n.value

    def storage(self):
        """(K, V) views of the whole pool, [max_blocks * bs, H, D]."""
        n = self.max_blocks * self.bs * self.H * self.D
        k = np.ctypeslib.as_array(self.lib.kvo_pool_k(self.p), shape=(n,))
        v = np.ctypeslib.as_array(self.lib.kvo_pool_v(self.p), shape=(n,))
        shape = (self.max_blocks * self.bs, self.H, self.D)
        return k.reshape(shape), v.reshape(shape)

    def attention(self, seq, q, Hq):
        k, v = self.storage()
        return gqa_attention_paged(q, k, v, self.block_table(seq), self.length(seq), self.bs, Hq, self.H, self.D)


class RefPool:
    """The reference's own KVBlockPool, through oracle/_ref/libs1ref.so."""

    def __init__(self, num_heads, head_dim, max_blocks, block_size=16):
        self.lib = _load_ref()
        self.H, self.D, self.max_blocks, self.bs = num_heads, head_dim, max_blocks, block_size
        self.p = self.lib.ref_pool_new(num_heads, head_dim, max_blocks, block_size)

    def __del__(self):
        if getattr(self, "p", None):
            self.lib.ref_pool_free(self.p)
            self.p = None

    def append(self, seq, k, v):
        k, v = _f32(k), _f32(v)
        return self.lib.ref_append(self.p, seq, _fp(k), _fp(v), k.shape[0], self.H, self.D)

    def length(self, seq):
        return int(self.lib.ref_length(self.p, seq))

    def remove(self, seq):
        return self.lib.ref_remove(self.p, seq)

    def truncate(self, seq, keep):
        return self.lib.ref_truncate(self.p, seq, keep)

    def get(self, seq, which):
        out = np.empty((self.length(seq), self.H, self.D), np.float32)
        if self.lib.ref_get(self.p, seq, which, _fp(out)) != 0:
            raise RuntimeError("KVBlockPool: Sequence ID not found")
        return out

    def block_table(self, seq):
        cap = self.max_blocks + 1
        out = np.zeros(cap, np.int32)
        n = i64()
        if self.lib.ref_block_table(self.p, seq, _fp(out), cap, C.byref(n)) != 0:
            return None
        return out[: n.value].copy()

    def storage(self, any_seq):
        n = self.max_blocks * self.bs * self.H * self.D
        shape = (self.max_blocks * self.bs, self.H, self.D)
        k = np.ctypeslib.as_array(self.lib.ref_pool_base(self.p, any_seq, 0), shape=(n,)).reshape(shape)
        v = np.ctypeslib.as_array(self.lib.ref_pool_base(self.p, any_seq, 1), shape=(n,)).reshape(shape)
        return k, v

    def attention(self, seq, q, Hq):
        q = _f32(q)
        out = np.empty((q.shape[0], Hq, self.D), np.float32)
        if self.lib.ref_gqa_attention_paged(self.p, seq, _fp(q), q.shape[0], Hq, self.H, self.D, _fp(out)) != 0:
            raise RuntimeError("Sequence ID not found")
        return out


def ref_apply_rope(x, start_pos=0):
    lib = _load_ref()
    x = _f32(x)
    out = np.empty_like(x)
    if x.ndim == 3:
        lib.ref_apply_rope(_fp(x), x.shape[0], x.shape[1], x.shape[2], start_pos, _fp(out))
    else:
        lib.ref_apply_rope(_fp(x), x.shape[0], 0, x.shape[1], start_pos, _fp(out))
    return out


def ref_rmsnorm(x, w, eps=1e-6):
    lib = _load_ref()
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    lib.ref_rmsnorm(_fp(x), x.size // x.shape[-1], x.shape[-1], _fp(w), eps, _fp(out))
    return out


def ref_gqa_attention(q, k, v, Hq, Hkv, D):
    lib = _load_ref()
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty((q.shape[0], Hq, D), np.float32)
    lib.ref_gqa_attention(_fp(q), _fp(k), _fp(v), q.shape[0], k.shape[0], Hq, Hkv, D, _fp(out))
    return out


def ref_decode_batch(pools, seqs, q, Hq, Hkv, D, n_threads):
    """q: [n_layers, n_seqs, Hq, D]; one GQA_attention_paged per (layer, seq)."""
    lib = _load_ref()
    q = _f32(q)
    arr = (vp * len(pools))(*[p.p for p in pools])
    s = np.ascontiguousarray(seqs, dtype=np.uint64)
    out = np.empty_like(q)
    lib.ref_decode_batch(arr, len(pools), _fp(s), s.size, _fp(q), Hq, Hkv, D, n_threads, _fp(out))
    return out
