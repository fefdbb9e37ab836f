"""Python binding of libs1kv (the C ABI in include/s1kv.h).

Two layers:

* ``Pool`` / ``Batch`` -- thin wrappers of the C ABI: a multi-layer device
  pool, host bookkeeping calls, and the batched decode/prefill step.  Device
  tensors are torch CUDA tensors; kernels run on torch's current stream.
* ``KVBlockPool`` / ``KVView`` / ``gqa_attention_paged`` / ``gqa_attention``
  / ``apply_rope`` -- the s1-infer interface (include/infer/kv_block_pool.h,
  include/nn/attention.h, include/nn/RoPE.h) with the same names, argument
  meaning and error behaviour (RuntimeError where the reference throws
  std::runtime_error).

There is no CPU path: importing works anywhere, but every call that needs
the engine loads libs1kv.so and raises if it or a CUDA device is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from collections import namedtuple

import numpy as np

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "lib", "libs1kv.so")

OK, ENOBLOCKS, ENOSEQ, EINVAL, ECUDA, ETIMEOUT, ENOMEM, EDEVICE = range(8)
DTYPE_F32, DTYPE_BF16 = 0, 1
POOL_HOST_ONLY = 1
K, V = 0, 1

i32, i64, u64, f32, vp = C.c_int32, C.c_int64, C.c_uint64, C.c_float, C.c_void_p
P = C.POINTER


class S1KVError(RuntimeError):
    """A non-OK status from libs1kv.  Subclasses RuntimeError like the
    reference's std::runtime_error."""

    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


class PoolDesc(C.Structure):
    _fields_ = [("num_layers", i32), ("num_kv_heads", i32), ("head_dim", i32), ("block_size", i32),
                ("max_blocks", i64), ("dtype", i32), ("max_seqs", i32), ("max_seq_len", i64),
                ("rope_theta", f32), ("flags", i32), ("initial_free_list", P(i32))]


class PrefixInfo(C.Structure):
    _fields_ = [("version", i32), ("num_layers", i32), ("num_kv_heads", i32), ("head_dim", i32), ("block_size", i32),
                ("dtype", i32), ("has_tokens", i32), ("n_tokens", i64), ("rope_theta", f32)]


def prefix_file_info(path):
    """Header of a format-1 prefix file, after checking its size and checksum
    (host only)."""
    info = PrefixInfo()
    check(lib().s1kv_prefix_file_info(str(path).encode(), C.byref(info)))
    return {f: getattr(info, f) for f, _ in PrefixInfo._fields_}


class PoolStats(C.Structure):
    _fields_ = [("num_free", i64), ("num_lru", i64), ("num_cached", i64), ("num_seqs", i64),
                ("cow_copies", i64), ("evictions", i64), ("device_bytes", i64)]


# name: (restype, argtypes) for every symbol of include/s1kv.h
SIGNATURES = {
    "s1kv_last_error": (C.c_char_p, []),
    "s1kv_status_str": (C.c_char_p, [C.c_int]),
    "s1kv_pool_create": (C.c_int, [P(PoolDesc), C.c_int, P(vp)]),
    "s1kv_pool_destroy": (C.c_int, [vp]),
    "s1kv_pool_get_desc": (C.c_int, [vp, P(PoolDesc)]),
    "s1kv_pool_stats_get": (C.c_int, [vp, P(PoolStats)]),
    "s1kv_pool_storage": (C.c_int, [vp, i32, P(vp), P(vp)]),
    "s1kv_pool_read": (C.c_int, [vp, i32, i32, i64, i64, vp]),
    "s1kv_pool_check": (C.c_int, [vp, P(i32)]),
    "s1kv_seq_reserve": (C.c_int, [vp, u64, i64, P(i32), P(i64)]),
    "s1kv_seq_length": (i64, [vp, u64]),
    "s1kv_seq_exists": (C.c_int, [vp, u64]),
    "s1kv_seq_remove": (C.c_int, [vp, u64]),
    "s1kv_seq_truncate": (C.c_int, [vp, u64, i64]),
    "s1kv_seq_fork": (C.c_int, [vp, u64, u64, i64]),
    "s1kv_block_table": (C.c_int, [vp, u64, P(i32), i64, P(i64)]),
    "s1kv_block_refcount": (C.c_int, [vp, i32, P(i32)]),
    "s1kv_free_list": (C.c_int, [vp, P(i32), i64, P(i64)]),
    "s1kv_lru_list": (C.c_int, [vp, P(i32), i64, P(i64)]),
    "s1kv_prefix_insert": (C.c_int, [vp, u64, P(i32), i64, P(i64)]),
    "s1kv_prefix_match": (C.c_int, [vp, u64, P(i32), i64, P(i64)]),
    "s1kv_block_hash": (u64, [u64, P(i32), i64]),
    "s1kv_prefix_save": (C.c_int, [vp, u64, C.c_char_p]),
    "s1kv_prefix_load": (C.c_int, [vp, u64, i64, C.c_char_p]),
    "s1kv_flush": (C.c_int, [vp, vp]),
    "s1kv_append": (C.c_int, [vp, i32, vp, vp, vp, i64, vp]),
    "s1kv_rope_append": (C.c_int, [vp, i32, vp, vp, i32, vp, vp, vp, vp, i64, i64, vp]),
    "s1kv_device_check": (C.c_int, [C.c_int, P(i32)]),
    "s1kv_apply_rope": (C.c_int, [vp, vp, i64, i64, i32, i32, f32, vp]),
    "s1kv_gather": (C.c_int, [vp, i32, u64, i32, vp, vp]),
    "s1kv_cow_copy": (C.c_int, [vp, vp, vp, i64, vp]),
    "s1kv_attention": (C.c_int, [vp, i32, P(u64), P(i32), i32, vp, vp, i32, vp]),
    "s1kv_attention_contig": (C.c_int, [vp, vp, vp, i64, i64, i32, i32, i32, vp, vp]),
    "s1kv_decode_attention_noalloc": (C.c_int, [vp, vp, i32, i64, i32, i32, i32, vp, i32, vp, i32, i32, vp, vp,
                                                i32, vp]),
    "s1kv_batch_begin": (C.c_int, [vp, P(u64), P(i32), P(i32), i32, vp, P(vp)]),
    "s1kv_batch_sizes": (C.c_int, [vp, P(i64), P(i64)]),
    "s1kv_batch_rope_append": (C.c_int, [vp, i32, vp, vp, i32, vp, vp, vp]),
    "s1kv_prefix_save_v1": (C.c_int, [vp, u64, P(i32), C.c_char_p]),
    "s1kv_prefix_file_info": (C.c_int, [C.c_char_p, vp]),
    "s1kv_prefix_load_v1": (C.c_int, [vp, u64, C.c_char_p, i32, P(i64)]),
    "s1kv_exchange_create": (C.c_int, [C.c_int, i32, i32, i64, P(vp)]),
    "s1kv_exchange_handle": (C.c_int, [vp, vp]),
    "s1kv_exchange_open": (C.c_int, [vp, vp]),
    "s1kv_exchange_wait_copy": (C.c_int, [vp, C.c_uint32, i32, i32, i32, i32, i32, vp, vp]),
    "s1kv_exchange_base": (vp, [vp]),
    "s1kv_exchange_open_local": (C.c_int, [vp, vp]),
    "s1kv_exchange_buffer": (vp, [vp, C.c_uint32]),
    "s1kv_exchange_wait": (C.c_int, [vp, C.c_uint32, vp]),
    "s1kv_exchange_destroy": (C.c_int, [vp]),
    "s1kv_batch_attention_exchange": (C.c_int, [vp, i32, vp, i32, vp, i32, i32, C.c_uint32, vp]),
    "s1kv_batch_norm_rope_append": (C.c_int, [vp, i32, vp, vp, i32, vp, vp, vp, vp, f32, vp]),
    "s1kv_debug_div_check": (C.c_int, [vp, i64, vp, i64, vp, vp]),
    "s1kv_batch_append": (C.c_int, [vp, i32, vp, vp, vp]),
    "s1kv_batch_attention": (C.c_int, [vp, i32, vp, vp, i32, vp]),
    "s1kv_batch_layer_host": (C.c_int, [vp, i32, vp, vp, vp, vp, i32, vp]),
    "s1kv_batch_end": (C.c_int, [vp, vp]),
    "s1kv_quantize_rows": (C.c_int, [vp, i64, i64, vp, vp, vp]),
    "s1kv_matmul_int8": (C.c_int, [vp, i64, i64, vp, vp, i64, vp, vp]),
    "s1kv_matmul_int8_group": (C.c_int, [vp, i64, i64, i32, vp, vp, vp, vp, vp]),
    "s1kv_launch_count": (i64, []),
    "s1kv_batch_plan": (C.c_int, [vp, P(i32), P(i64)]),
}

_lib = None


def lib():
    """Load libs1kv.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libs1kv.so not built ({LIB_PATH}); run s1-infer_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status):
    if status != OK:
        L = lib()
        raise S1KVError(status, L.s1kv_last_error().decode() or L.s1kv_status_str(status).decode())
    return status


def _i32p(a):
    return a.ctypes.data_as(P(i32)) if a is not None else None


def _stream():
    import torch
    return vp(torch.cuda.current_stream().cuda_stream)


def _dptr(t):
    return vp(t.data_ptr()) if t is not None else None


def _cuda_f32(x, device):
    """float32 contiguous CUDA tensor on `device` (None = current device)."""
    import torch
    t = torch.as_tensor(x)
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    return t.to(device=dev, dtype=torch.float32).contiguous()


def launch_count():
    return int(lib().s1kv_launch_count())


def device_check(device=0):
    """Reads and clears the device error word; raises S1KVError if set."""
    f = i32()
    check(lib().s1kv_device_check(device, C.byref(f)))
    return f.value


# ==================================================================== Pool ==

class Pool:
    """A device-resident block pool of ``num_layers`` layers sharing one block
    table per sequence (include/s1kv.h)."""

    def __init__(self, num_layers, num_kv_heads, head_dim, max_blocks, block_size=16, dtype="f32", device=None,
                 max_seqs=1024, max_seq_len=0, rope_theta=1.0e6, initial_free_list=None, host_only=False):
        """device None = torch's current CUDA device (0 for a host-only pool)."""
        self.L = lib()
        if device is None:
            if host_only:
                device = 0
            else:
                import torch
                device = torch.cuda.current_device()
        self.num_layers, self.Hkv, self.D = num_layers, num_kv_heads, head_dim
        self.max_blocks, self.bs = max_blocks, block_size
        self.dtype = DTYPE_F32 if dtype in ("f32", "fp32", "float32", DTYPE_F32) else DTYPE_BF16
        self.device = device
        d = PoolDesc(num_layers, num_kv_heads, head_dim, block_size, max_blocks, self.dtype, max_seqs, max_seq_len,
                     rope_theta, POOL_HOST_ONLY if host_only else 0, None)
        fl = None
        if initial_free_list is not None:
            fl = np.ascontiguousarray(initial_free_list, dtype=np.int32)
            d.initial_free_list = _i32p(fl)
        h = vp()
        check(self.L.s1kv_pool_create(C.byref(d), device, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.L.s1kv_pool_destroy(self.h)
            self.h = None

    __del__ = close

    # ---- bookkeeping ----
    def reserve(self, seq, n):
        slots = np.zeros(max(n, 1), np.int32)
        done = i64()
        st = self.L.s1kv_seq_reserve(self.h, seq, n, _i32p(slots), C.byref(done))
        return st, slots[: done.value].copy()

    def length(self, seq):
        return int(self.L.s1kv_seq_length(self.h, seq))

    def exists(self, seq):
        return bool(self.L.s1kv_seq_exists(self.h, seq))

    def remove(self, seq):
        check(self.L.s1kv_seq_remove(self.h, seq))

    def truncate(self, seq, keep):
        check(self.L.s1kv_seq_truncate(self.h, seq, keep))

    def fork(self, src, dst, n):
        check(self.L.s1kv_seq_fork(self.h, src, dst, n))

    def block_table(self, seq):
        n = i64()
        check(self.L.s1kv_block_table(self.h, seq, None, 0, C.byref(n)))
        out = np.zeros(max(n.value, 1), np.int32)
        check(self.L.s1kv_block_table(self.h, seq, _i32p(out), n.value, C.byref(n)))
        return out[: n.value]

    def refcount(self, block):
        r = i32()
        check(self.L.s1kv_block_refcount(self.h, block, C.byref(r)))
        return r.value

    def refcounts(self):
        return np.array([self.refcount(b) for b in range(self.max_blocks)], np.int32)

    def free_list(self):
        n = i64()
        check(self.L.s1kv_free_list(self.h, None, 0, C.byref(n)))
        out = np.zeros(max(n.value, 1), np.int32)
        check(self.L.s1kv_free_list(self.h, _i32p(out), n.value, C.byref(n)))
        return out[: n.value]

    def lru_list(self):
        n = i64()
        check(self.L.s1kv_lru_list(self.h, None, 0, C.byref(n)))
        out = np.zeros(max(n.value, 1), np.int32)
        check(self.L.s1kv_lru_list(self.h, _i32p(out), n.value, C.byref(n)))
        return out[: n.value]

    def stats(self):
        s = PoolStats()
        check(self.L.s1kv_pool_stats_get(self.h, C.byref(s)))
        return {f: getattr(s, f) for f, _ in PoolStats._fields_}

    def prefix_insert(self, seq, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        n = i64()
        check(self.L.s1kv_prefix_insert(self.h, seq, _i32p(t), t.size, C.byref(n)))
        return n.value

    def prefix_match(self, dst, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        n = i64()
        check(self.L.s1kv_prefix_match(self.h, dst, _i32p(t), t.size, C.byref(n)))
        return n.value

    def prefix_save(self, seq, path):
        check(self.L.s1kv_prefix_save(self.h, seq, str(path).encode()))

    def prefix_save_v1(self, seq, path, tokens=None):
        t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
        check(self.L.s1kv_prefix_save_v1(self.h, seq, _i32p(t), str(path).encode()))

    def prefix_load_v1(self, seq, path, register=False):
        n = i64()
        check(self.L.s1kv_prefix_load_v1(self.h, seq, str(path).encode(), int(register), C.byref(n)))
        return n.value

    def prefix_load(self, seq, n_tokens, path):
        check(self.L.s1kv_prefix_load(self.h, seq, n_tokens, str(path).encode()))

    # ---- device ----
    def check_device(self):
        f = i32()
        check(self.L.s1kv_pool_check(self.h, C.byref(f)))
        return f.value

    def flush(self):
        check(self.L.s1kv_flush(self.h, _stream()))

    def read_storage(self, layer, which, slot0=0, n_slots=None):
        """Raw storage rows [slot0, slot0+n_slots) as numpy (float32 or the
        uint16 bf16 bits)."""
        n_slots = self.max_blocks * self.bs - slot0 if n_slots is None else n_slots
        dt = np.float32 if self.dtype == DTYPE_F32 else np.uint16
        out = np.empty((n_slots, self.Hkv, self.D), dt)
        check(self.L.s1kv_pool_read(self.h, layer, which, slot0, n_slots, out.ctypes.data_as(vp)))
        return out

    def append(self, layer, k, v, slots):
        import torch
        k, v = _cuda_f32(k, self.device), _cuda_f32(v, self.device)
        s = torch.as_tensor(slots, dtype=torch.int32).to(self.device)
        check(self.L.s1kv_append(self.h, layer, _dptr(k), _dptr(v), _dptr(s), k.shape[0], _stream()))

    def rope_append(self, layer, k, v, slots, pos, q=None):
        import torch
        k, v = _cuda_f32(k, self.device), _cuda_f32(v, self.device)
        s = torch.as_tensor(slots, dtype=torch.int32).to(self.device)
        p = torch.as_tensor(pos, dtype=torch.int32).to(self.device)
        q_in = _cuda_f32(q, self.device) if q is not None else None
        q_out = torch.empty_like(q_in) if q_in is not None else None
        max_pos = int(np.max(np.asarray(pos))) + 1 if len(pos) else 0
        check(self.L.s1kv_rope_append(self.h, layer, _dptr(q_in), _dptr(q_out), q_in.shape[1] if q_in is not None else 0,
                                      _dptr(k), _dptr(v), _dptr(s), _dptr(p), k.shape[0], max_pos, _stream()))
        return q_out

    def gather(self, layer, seq, which):
        import torch
        out = torch.empty((self.length(seq), self.Hkv, self.D), dtype=torch.float32, device=self.device)
        check(self.L.s1kv_gather(self.h, layer, seq, which, _dptr(out), _stream()))
        return out

    def cow_copy(self, src, dst):
        import torch
        s = torch.as_tensor(src, dtype=torch.int32).to(self.device)
        d = torch.as_tensor(dst, dtype=torch.int32).to(self.device)
        check(self.L.s1kv_cow_copy(self.h, _dptr(s), _dptr(d), s.numel(), _stream()))

    def attention(self, layer, seqs, q_lens, q, n_q_heads):
        import torch
        seqs = np.ascontiguousarray(seqs, dtype=np.uint64)
        ql = np.ascontiguousarray(q_lens, dtype=np.int32)
        q = _cuda_f32(q, self.device)
        out = torch.empty_like(q)
        check(self.L.s1kv_attention(self.h, layer, seqs.ctypes.data_as(P(u64)), _i32p(ql), seqs.size, _dptr(q),
                                    _dptr(out), n_q_heads, _stream()))
        return out

    def batch(self, seqs, n_append=None, q_lens=None):
        return Batch(self, seqs, n_append, q_lens)


class Batch:
    """One step of many sequences (s1kv_batch_*).  Use as a context manager
    or call end()."""

    def __init__(self, pool, seqs, n_append=None, q_lens=None):
        self.pool, self.L = pool, pool.L
        self.seqs = np.ascontiguousarray(seqs, dtype=np.uint64)
        self.na = None if n_append is None else np.ascontiguousarray(n_append, dtype=np.int32)
        self.ql = None if q_lens is None else np.ascontiguousarray(q_lens, dtype=np.int32)
        h = vp()
        check(self.L.s1kv_batch_begin(pool.h, self.seqs.ctypes.data_as(P(u64)), _i32p(self.na), _i32p(self.ql),
                                      self.seqs.size, _stream(), C.byref(h)))
        self.h = h
        nt, nr = i64(), i64()
        check(self.L.s1kv_batch_sizes(h, C.byref(nt), C.byref(nr)))
        self.n_tokens, self.n_rows = nt.value, nr.value

    def plan(self):
        s, n = i32(), i64()
        check(self.L.s1kv_batch_plan(self.h, C.byref(s), C.byref(n)))
        return s.value, n.value

    def rope_append(self, layer, k, v, q=None, q_out=None):
        """k, v: [n_tokens, Hkv, D] fp32 CUDA; q (optional) [n_rows, Hq, D] is
        rotated into q_out (allocated when not given)."""
        import torch
        if q is not None and q_out is None:
            q_out = torch.empty_like(q)
        check(self.L.s1kv_batch_rope_append(self.h, layer, _dptr(q), _dptr(q_out), q.shape[1] if q is not None else 0,
                                            _dptr(k), _dptr(v), _stream()))
        return q_out

    def norm_rope_append(self, layer, k, v, k_norm_weight, q=None, q_norm_weight=None, eps=1e-6, q_out=None):
        """q/k RMSNorm + RoPE + append in one kernel: k, v [n_tokens, Hkv, D]
        and q [n_rows, Hq, D] are the raw projection outputs; the norm
        weights are fp32 CUDA [D].  Returns the normalised, rotated q."""
        import torch
        if q is not None and q_out is None:
            q_out = torch.empty_like(q)
        check(self.L.s1kv_batch_norm_rope_append(self.h, layer, _dptr(q), _dptr(q_out),
                                                 q.shape[1] if q is not None else 0, _dptr(q_norm_weight), _dptr(k),
                                                 _dptr(v), _dptr(k_norm_weight), eps, _stream()))
        return q_out

    def append(self, layer, k, v):
        check(self.L.s1kv_batch_append(self.h, layer, _dptr(k), _dptr(v), _stream()))

    def attention(self, layer, q, out=None):
        import torch
        if out is None:
            out = torch.empty_like(q)
        check(self.L.s1kv_batch_attention(self.h, layer, _dptr(q), _dptr(out), q.shape[1], _stream()))
        return out

    def layer_host(self, layer, h_q, h_k, h_v, h_out, n_q_heads):
        """End-to-end step of one layer from host (pinned) tensors."""
        check(self.L.s1kv_batch_layer_host(self.h, layer, _dptr(h_q), _dptr(h_k), _dptr(h_v), _dptr(h_out),
                                           n_q_heads, _stream()))

    def end(self):
        if getattr(self, "h", None):
            check(self.L.s1kv_batch_end(self.h, _stream()))
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.end()


# ============================================ s1-infer reference interface ==

# struct KVView (include/infer/kv_block_pool.h:6-11): base is the device
# address of the layer's K or V storage; block_table a host copy.
KVView = namedtuple("KVView", ["base", "block_table", "block_size", "total_tokens", "pool", "seq", "which"])


class KVBlockPool:
    """KVBlockPool(num_heads, head_dim, max_blocks, block_size=16)
    (include/infer/kv_block_pool.h:32), backed by a one-layer device pool.
    Tensors are [tokens, num_heads, head_dim] fp32 (numpy or torch)."""

    def __init__(self, num_heads, head_dim, max_blocks, block_size=16, device=None, dtype="f32", initial_free_list=None):
        self.pool = Pool(1, num_heads, head_dim, max_blocks, block_size, dtype=dtype, device=device,
                         initial_free_list=initial_free_list)
        self.num_heads, self.head_dim, self.block_size = num_heads, head_dim, block_size

    def append(self, sequence_id, k, v):
        """KVBlockPool::append (kv_block_pool.cpp:20-65).  On exhaustion the
        tokens that fit are stored, then RuntimeError is raised, as the
        reference throws after partial progress (:36-38)."""
        import torch
        k = _cuda_f32(k, self.pool.device)
        v = _cuda_f32(v, self.pool.device)
        T = k.shape[0]
        st, slots = self.pool.reserve(sequence_id, T)
        if len(slots):
            n = len(slots)
            self.pool.append(0, k[:n].reshape(n, self.num_heads, self.head_dim),
                             v[:n].reshape(n, self.num_heads, self.head_dim), slots)
            torch.cuda.current_stream().synchronize()
        check(st)

    def get_k(self, sequence_id):
        return self.pool.gather(0, sequence_id, K)

    def get_v(self, sequence_id):
        return self.pool.gather(0, sequence_id, V)

    def length(self, sequence_id):
        return self.pool.length(sequence_id)

    def remove(self, sequence_id):
        self.pool.remove(sequence_id)

    def truncate(self, sequence_id, keep_length):
        self.pool.truncate(sequence_id, keep_length)

    def _view(self, sequence_id, which):
        if not self.pool.exists(sequence_id):
            raise S1KVError(ENOSEQ, "Sequence ID not found")
        kb, vb = vp(), vp()
        check(self.pool.L.s1kv_pool_storage(self.pool.h, 0, C.byref(kb), C.byref(vb)))
        return KVView((kb if which == K else vb).value, self.pool.block_table(sequence_id), self.block_size,
                      self.pool.length(sequence_id), self.pool, sequence_id, which)

    def get_k_view(self, sequence_id):
        return self._view(sequence_id, K)

    def get_v_view(self, sequence_id):
        return self._view(sequence_id, V)


def gqa_attention_paged(Q, k_view, v_view, num_q_heads, num_kv_heads, head_dim):
    """GQA_attention_paged (include/nn/attention.h:10).  Q [q_len, Hq, D]."""
    pool = k_view.pool
    Q = _cuda_f32(Q, pool.device)
    if k_view.seq != v_view.seq or k_view.pool is not v_view.pool:
        raise S1KVError(EINVAL, "k_view and v_view must view the same sequence")
    if num_kv_heads != pool.Hkv or head_dim != pool.D:
        raise S1KVError(EINVAL, "head shape does not match the pool")
    return pool.attention(0, [k_view.seq], [Q.shape[0]], Q.reshape(Q.shape[0], num_q_heads, head_dim), num_q_heads)


def gqa_attention(Q, Kc, Vc, num_q_heads, num_kv_heads, head_dim, device=None):
    """GQA_attention over contiguous K/V (include/nn/attention.h:8)."""
    import torch
    Q, Kc, Vc = _cuda_f32(Q, device), _cuda_f32(Kc, device), _cuda_f32(Vc, device)
    out = torch.empty((Q.shape[0], num_q_heads, head_dim), dtype=torch.float32, device=Q.device)
    check(lib().s1kv_attention_contig(_dptr(Q), _dptr(Kc), _dptr(Vc), Q.shape[0], Kc.shape[0], num_q_heads,
                                      num_kv_heads, head_dim, _dptr(out), _stream()))
    return out


def apply_rope(x, start_pos=0, theta=1.0e6, device=None):
    """apply_rope(input, start_pos) (include/nn/RoPE.h:4): [T, H, D] or [T, D]."""
    import torch
    x = _cuda_f32(x, device)
    shape = x.shape
    x3 = x.reshape(shape[0], -1, shape[-1])
    out = torch.empty_like(x3)
    with torch.cuda.device(x.device):
        check(lib().s1kv_apply_rope(_dptr(x3), _dptr(out), start_pos, x3.shape[0], x3.shape[1], x3.shape[2], theta,
                                    _stream()))
    return out.reshape(shape)


# ============================================== int8 projections ==========
# quantize_tensor / dequantize / matmul_quantized (include/core/
# quantized_tensor.h:7-23): the weights either side of the KV path, int8 with
# one scale per row k of the pre-transposed [K, N] weight.

class QuantizedTensor:
    """struct QuantizedTensor (include/core/quantized_tensor.h:7-12): data
    int8 [rows, cols] and scales fp32 [rows], both on the GPU."""

    def __init__(self, data, scales):
        self.data, self.scales = data, scales
        self.rows, self.cols = int(data.shape[0]), int(data.shape[1])


def quantize_tensor(t, device=None):
    """quantize_tensor (src/quantized_tensor.cpp:9-47): a [rows, cols] float
    tensor to int8 with scale max|row| / 127 per row (1 for a zero row) and
    round(value / scale), ties away from zero; bit-exact."""
    import torch
    w = _cuda_f32(t, device)
    if w.dim() != 2:
        raise S1KVError(EINVAL, "quantize_tensor needs a 2-D tensor")
    q = torch.empty(w.shape, dtype=torch.int8, device=w.device)
    sc = torch.empty((w.shape[0],), dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        check(lib().s1kv_quantize_rows(_dptr(w), w.shape[0], w.shape[1], _dptr(q), _dptr(sc), _stream()))
    return QuantizedTensor(q, sc)


def dequantize(qt, row, col):
    """dequantize (src/quantized_tensor.cpp:49-57): q[row, col] * scale[row]."""
    import numpy as np
    return float(np.float32(int(qt.data[row, col])) * np.float32(float(qt.scales[row])))


def matmul_quantized(x, w, out=None):
    """matmul_quantized (src/quantized_tensor.cpp:102-122): x [M, K] float
    times the quantized [K, N] weight -> [M, N] fp32 (within 2e-5 of the
    output scale of the reference's sequential sum)."""
    import torch
    xd = _cuda_f32(x, w.data.device.index)
    if xd.dim() != 2 or xd.shape[1] != w.rows:
        raise S1KVError(EINVAL, "matmul_quantized: x must be [M, %d]" % w.rows)
    if out is None:
        out = torch.empty((xd.shape[0], w.cols), dtype=torch.float32, device=xd.device)
    with torch.cuda.device(xd.device):
        check(lib().s1kv_matmul_int8(_dptr(xd), xd.shape[0], w.rows, _dptr(w.data), _dptr(w.scales), w.cols,
                                     _dptr(out), _stream()))
    return out


def matmul_quantized_group(x, ws, outs=None):
    """Products of one x with up to 4 quantized weights of the same K in one
    launch (q/k/v, gate/up): the same results as matmul_quantized on each."""
    import torch
    dev = ws[0].data.device.index
    xd = _cuda_f32(x, dev)
    if xd.dim() != 2 or any(w.rows != xd.shape[1] for w in ws):
        raise S1KVError(EINVAL, "matmul_quantized_group: x must be [M, K] with K the weights' rows")
    if outs is None:
        outs = [torch.empty((xd.shape[0], w.cols), dtype=torch.float32, device=xd.device) for w in ws]
    n = len(ws)
    qa = (vp * n)(*[w.data.data_ptr() for w in ws])
    sa = (vp * n)(*[w.scales.data_ptr() for w in ws])
    na = (i64 * n)(*[w.cols for w in ws])
    oa = (vp * n)(*[o.data_ptr() for o in outs])
    with torch.cuda.device(xd.device):
        check(lib().s1kv_matmul_int8_group(_dptr(xd), xd.shape[0], xd.shape[1], n, qa, sa, na, oa, _stream()))
    return outs


# ================================================ KV-head-sharded serving ==
# Long-context requests are split across GPUs by KV head: rank r of `world`
# keeps a pool holding only KV heads [kv_lo, kv_hi) of every token (and runs
# the query heads of those groups); after each layer's attention one
# all-gather over NVLink gives every rank the outputs of all heads.  No
# reference counterpart: s1-infer runs on one host thread.

def head_shard(world, rank, num_kv_heads, num_q_heads):
    """(kv_lo, kv_hi, q_lo, q_hi): the KV heads and query heads rank `rank`
    of `world` owns.  Whole GQA groups stay together (query head h reads KV
    head h // (Hq / Hkv)), so every rank runs the unchanged kernels on a
    pool of num_kv_heads / world heads."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if num_kv_heads % world or num_q_heads % num_kv_heads:
        raise ValueError(f"{num_kv_heads} KV heads / {num_q_heads} query heads do not split over {world} ranks")
    kv = num_kv_heads // world
    q = num_q_heads // world
    return rank * kv, (rank + 1) * kv, rank * q, (rank + 1) * q


def gather_heads(out_local, world, group=None, buf=None):
    """All-gather of per-rank attention outputs [B, Hq/world, D] into the
    token-major [B, Hq, D] every rank needs for the output projection: one
    collective (NCCL all_gather_into_tensor over NVLink on GPUs, gloo on
    CPU) into a head-major buffer [world, B, Hq/world, D], then the
    head-major to token-major reorder.  `buf` (optional) is that buffer."""
    import torch
    import torch.distributed as dist
    B, hq_l, D = out_local.shape
    if world == 1:
        return out_local
    src = out_local.contiguous()
    if buf is None:
        buf = torch.empty((world, B, hq_l, D), dtype=src.dtype, device=src.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, src, group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), src, group=group)
    return buf.transpose(0, 1).reshape(B, world * hq_l, D)


class _DeviceArray:
    """__cuda_array_interface__ view of device memory owned elsewhere (fp32;
    strides in bytes, None for contiguous)."""

    def __init__(self, ptr, shape, strides=None):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": strides}


class PeerExchange:
    """Fused output exchange of a KV-head-sharded job (s1kv_exchange_*): the
    decode kernels store each finished element, tagged with the layer's
    epoch in one 64-bit word, into every rank's token-major buffer
    [rows, heads_total, head_dim] over NVLink; wait(epoch) makes the stream
    wait (bounded) until all ranks' words carry the epoch.  Epochs start at
    1.  The CUDA IPC handles are exchanged once through torch.distributed."""

    def __init__(self, rank, world, rows, heads_total, head_dim, device=None, group=None, local=False):
        import torch
        self.L = lib()
        self.rank, self.world = rank, world
        self.shape = (rows, heads_total, head_dim)
        dev = torch.cuda.current_device() if device is None else device
        h = vp()
        check(self.L.s1kv_exchange_create(dev, rank, world, rows * heads_total * head_dim, C.byref(h)))
        self.h = h
        if world > 1 and not local:
            import torch.distributed as dist
            mine = (C.c_char * 64)()
            check(self.L.s1kv_exchange_handle(h, mine))
            handles = [None] * world
            dist.all_gather_object(handles, bytes(mine), group=group)
            arr = (C.c_char * (64 * world)).from_buffer_copy(b"".join(handles))
            check(self.L.s1kv_exchange_open(h, arr))

    @staticmethod
    def open_local(exchanges):
        """Opens the exchanges of all ranks of one process (created with
        local=True, in rank order) on each other's device memory instead of
        CUDA IPC handles (s1kv_exchange_open_local)."""
        L = lib()
        bases = (vp * len(exchanges))(*[L.s1kv_exchange_base(e.h) for e in exchanges])
        for e in exchanges:
            check(L.s1kv_exchange_open_local(e.h, bases))

    def attention(self, batch, layer, q, head0, epoch):
        """Decode attention of this rank's query heads q [rows, Hq_local, D]
        (global heads head0 ..), published under `epoch`."""
        check(self.L.s1kv_batch_attention_exchange(batch.h, layer, _dptr(q), q.shape[1], self.h, head0, self.shape[1],
                                                   epoch, _stream()))

    def wait(self, epoch, force=False):
        """Makes the stream wait until every rank's words of `epoch` arrived.
        With one rank the stream order already covers it, so nothing is
        launched unless `force`."""
        if self.world > 1 or force:
            check(self.L.s1kv_exchange_wait(self.h, epoch, _stream()))

    def wait_copy(self, epoch, head0, n_heads, dst):
        """Waits for every rank's `epoch` (always launched, also with one
        rank) and copies heads [head0, head0 + n_heads) of the gathered
        output into dst [rows, n_heads, head_dim] in the same kernel."""
        rows, heads_total, D = self.shape
        check(self.L.s1kv_exchange_wait_copy(self.h, epoch, dst.shape[0], heads_total, D, head0, n_heads, _dptr(dst),
                                             _stream()))
        return dst

    def output(self, epoch, rows=None):
        """The gathered [rows, heads_total, head_dim] of `epoch` (a strided
        fp32 view of the value halves of the exchange's words; valid until
        the slot is reused two epochs later or the exchange is closed).  The
        two slots' tensors are made once: a decode loop calls this every
        layer."""
        import torch
        if not hasattr(self, "_slots"):
            rows, heads, D = self.shape
            strides = (heads * D * 8, D * 8, 8)
            self._slots = [torch.as_tensor(_DeviceArray(self.L.s1kv_exchange_buffer(self.h, e), self.shape, strides),
                                           device="cuda") for e in (0, 1)]
        t = self._slots[epoch & 1]
        return t if rows is None else t[:rows]

    def close(self):
        if getattr(self, "h", None):
            self._slots = None
            self.L.s1kv_exchange_destroy(self.h)
            self.h = None

    __del__ = close
