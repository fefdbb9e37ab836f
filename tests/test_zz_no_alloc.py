"""s1kv_decode_attention_noalloc: decode attention for callers that cannot
allocate device memory where attention runs (an inference-server plugin's
execution step, where the server owns all device memory; a decode loop
that must not block in or fail on the allocator).  Its scratch is a fixed
array inside the library.

Checked through the C ABI against the CPU oracle (GQA_attention_paged of
src/nn/attention.cpp:128-239 restated, on the same bf16-rounded K/V for
bf16 storage) and against the regular entry point (s1kv_attention, which
plans on the host and uses the pool's own scratch), for two calls in a row,
with the fp32 tolerance of the other parity tests; the second call must not
change the device's free memory.  Lengths outside [1, max_seq_len] must be
reported through s1kv_device_check.  This file is collected last so that a
failure here stops a `-x` run only after every other test has run."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-5  # max |out - ref| / max |ref|, as in test_gpu_parity.py


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def filled_pool(s1kv, oracle, torch, dtype, Hq, Hkv, D, ctx, seed):
    """A one-layer pool holding ctx[i] random tokens for sequence i, the
    oracle pool with the same free list and contents, and the device block
    tables [n_seqs][max_bps] of the pool."""
    bs = 16
    rng = np.random.default_rng(seed)
    seqs = list(range(len(ctx)))
    max_blocks = sum((c + bs) // bs for c in ctx) + 8
    order = rng.permutation(max_blocks).astype(np.int32)
    pool = s1kv.Pool(1, Hkv, D, max_blocks, bs, dtype=dtype, initial_free_list=order)
    op = oracle.Pool(Hkv, D, max_blocks, bs, free_order=order)
    ks = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    vs = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    with pool.batch(seqs, ctx, [0] * len(ctx)) as b:
        b.append(0, torch.from_numpy(np.concatenate(ks)).cuda(), torch.from_numpy(np.concatenate(vs)).cuda())
    for s, k, v in zip(seqs, ks, vs):
        if dtype == "bf16":
            k, v = oracle.bf16_round(k), oracle.bf16_round(v)
        assert op.append(s, k, v) == 0
    max_bps = max(len(pool.block_table(s)) for s in seqs)
    tables = np.zeros((len(seqs), max_bps), np.int32)
    for i, s in enumerate(seqs):
        t = pool.block_table(s)
        np.testing.assert_array_equal(t, op.block_table(s))
        tables[i, : len(t)] = t
    return pool, op, seqs, max_blocks, torch.from_numpy(tables).cuda(), rng


def clear_error_word(s1kv):
    try:
        s1kv.device_check(0)
    except s1kv.S1KVError:
        pass


def call_noalloc(s1kv, pool, dtype, max_blocks, Hkv, D, d_tables, d_lens, n, max_len, q, out, Hq, stream):
    L = s1kv.lib()
    kb, vb = C.c_void_p(), C.c_void_p()
    s1kv.check(L.s1kv_pool_storage(pool.h, 0, C.byref(kb), C.byref(vb)))
    code = s1kv.DTYPE_F32 if dtype == "f32" else s1kv.DTYPE_BF16
    return L.s1kv_decode_attention_noalloc(kb, vb, code, max_blocks * 16, Hkv, D, 16, C.c_void_p(d_tables.data_ptr()),
                                           d_tables.shape[1], C.c_void_p(d_lens.data_ptr()), n, max_len,
                                           C.c_void_p(q.data_ptr()), C.c_void_p(out.data_ptr()), Hq, stream)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("shape", [(32, 8, 128), (14, 2, 64)])
def test_noalloc_matches_oracle_and_regular_entry_point(s1kv, oracle, cuda, dtype, shape):
    torch = cuda
    Hq, Hkv, D = shape
    ctx = [1, 15, 16, 17, 300, 1000, 2500, 40, 129]
    pool, op, seqs, max_blocks, d_tables, rng = filled_pool(s1kv, oracle, torch, dtype, Hq, Hkv, D, ctx, Hq + D)
    d_lens = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    # a stream that does not synchronise with the legacy default stream
    stream = torch.cuda.Stream()
    clear_error_word(s1kv)
    for call in range(2):
        q_h = rng.standard_normal((len(seqs), Hq, D), dtype=np.float32)
        q = torch.from_numpy(q_h).cuda()
        out = torch.full_like(q, float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        with torch.cuda.stream(stream):
            st = call_noalloc(s1kv, pool, dtype, max_blocks, Hkv, D, d_tables, d_lens, len(seqs), max(ctx), q, out,
                              Hq, C.c_void_p(stream.cuda_stream))
        s1kv.check(st)
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        if call == 1:
            assert free_after == free_before, "the call took device memory"
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        ref = np.concatenate([op.attention(s, q_h[i:i + 1], Hq) for i, s in enumerate(seqs)])
        err = rel_err(got, ref)
        print(f"noalloc {dtype} {shape} call {call}: rel err vs oracle {err:.2e}")
        assert err <= TOL, (call, err)
        regular = pool.attention(0, seqs, [1] * len(seqs), q, Hq).cpu().numpy()
        assert rel_err(got, regular) <= TOL, (call, rel_err(got, regular))
    assert s1kv.device_check(0) == 0


def test_noalloc_reports_bad_lengths(s1kv, oracle, cuda):
    """A length of 0 and one above max_seq_len are refused by the call's own
    device-side plan (their rows read nothing past the table) and reported
    through s1kv_device_check, which then reads clear; the valid rows are
    still right."""
    torch = cuda
    Hq, Hkv, D = 32, 8, 128
    ctx = [100, 300, 50]
    pool, op, seqs, max_blocks, d_tables, rng = filled_pool(s1kv, oracle, torch, "f32", Hq, Hkv, D, ctx, 3)
    max_len = max(ctx)
    lens = [ctx[0], 0, max_len + 5]  # row 1 empty, row 2 beyond the bound (clamped to max_len)
    d_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q_h = rng.standard_normal((3, Hq, D), dtype=np.float32)
    q = torch.from_numpy(q_h).cuda()
    out = torch.zeros_like(q)
    clear_error_word(s1kv)
    st = call_noalloc(s1kv, pool, "f32", max_blocks, Hkv, D, d_tables, d_lens, 3, max_len, q, out, Hq,
                      C.c_void_p(torch.cuda.current_stream().cuda_stream))
    s1kv.check(st)
    flags = C.c_int32(0)
    st = s1kv.lib().s1kv_device_check(0, C.byref(flags))
    assert st == s1kv.EDEVICE and flags.value & 1, (st, flags.value)
    assert s1kv.device_check(0) == 0  # cleared
    ref0 = op.attention(seqs[0], q_h[0:1], Hq)
    assert rel_err(out[0:1].cpu().numpy(), ref0) <= TOL


def test_noalloc_rejects_sizes_beyond_its_scratch(s1kv, cuda):
    """The size check uses only the scalar arguments, so one small buffer
    stands in for every pointer."""
    torch = cuda
    L = s1kv.lib()
    pool = s1kv.Pool(1, 8, 128, 64, 16)
    kb, vb = C.c_void_p(), C.c_void_p()
    s1kv.check(L.s1kv_pool_storage(pool.h, 0, C.byref(kb), C.byref(vb)))
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    ptr = C.c_void_p(dummy.data_ptr())
    n, max_len = 4096, 1 << 20  # far more partial results than 8 MiB holds
    st = L.s1kv_decode_attention_noalloc(kb, vb, s1kv.DTYPE_F32, 64 * 16, 8, 128, 16, ptr, max_len // 16, ptr, n,
                                         max_len, ptr, ptr, 32, None)
    assert st == s1kv.EINVAL
    assert "8 MiB" in L.s1kv_last_error().decode()
