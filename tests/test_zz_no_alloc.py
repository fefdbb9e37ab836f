"""s1kv_decode_attention_noalloc: decode attention for callers that cannot
allocate device memory where attention runs (an inference-server plugin's
execution step, a decode loop that must not block in the allocator).  Its
scratch is a fixed array inside the library.

Checked through the C ABI against the regular entry point (s1kv_attention,
which plans on the host and uses the pool's own scratch) on the same pool,
for two calls in a row, with the fp32 tolerance of the other parity tests;
the second call must not change the device's free memory.  This file is
collected last so that a failure here stops a `-x` run only after every
other test has run."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-5  # max |out - ref| / max |ref|, as in test_gpu_parity.py


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("shape", [(32, 8, 128), (14, 2, 64)])
def test_noalloc_matches_regular_entry_point(s1kv, cuda, dtype, shape):
    torch = cuda
    L = s1kv.lib()
    Hq, Hkv, D = shape
    bs = 16
    rng = np.random.default_rng(Hq + D)
    ctx = [1, 15, 16, 17, 300, 1000, 2500, 40, 129]
    seqs = list(range(len(ctx)))
    max_blocks = sum((c + bs) // bs for c in ctx) + 8
    pool = s1kv.Pool(1, Hkv, D, max_blocks, bs, dtype=dtype, initial_free_list=rng.permutation(max_blocks))
    with pool.batch(seqs, ctx, [0] * len(ctx)) as b:
        k = torch.from_numpy(rng.standard_normal((sum(ctx), Hkv, D), dtype=np.float32)).cuda()
        v = torch.from_numpy(rng.standard_normal((sum(ctx), Hkv, D), dtype=np.float32)).cuda()
        b.append(0, k, v)

    max_bps = max(len(pool.block_table(s)) for s in seqs)
    tables = np.zeros((len(seqs), max_bps), np.int32)
    for i, s in enumerate(seqs):
        t = pool.block_table(s)
        tables[i, : len(t)] = t
    d_tables = torch.from_numpy(tables).cuda()
    d_lens = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    kb, vb = C.c_void_p(), C.c_void_p()
    s1kv.check(L.s1kv_pool_storage(pool.h, 0, C.byref(kb), C.byref(vb)))
    code = s1kv.DTYPE_F32 if dtype == "f32" else s1kv.DTYPE_BF16
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((len(seqs), Hq, D), dtype=np.float32)).cuda()
        out = torch.full_like(q, float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = L.s1kv_decode_attention_noalloc(kb, vb, code, max_blocks * bs, Hkv, D, bs,
                                             C.c_void_p(d_tables.data_ptr()), max_bps,
                                             C.c_void_p(d_lens.data_ptr()), len(seqs), max(ctx),
                                             C.c_void_p(q.data_ptr()), C.c_void_p(out.data_ptr()), Hq, stream)
        s1kv.check(st)
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        if call == 1:
            assert free_after == free_before, "the call took device memory"
        ref = pool.attention(0, seqs, [1] * len(seqs), q, Hq)
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, ref.cpu().numpy()) <= TOL, (call, rel_err(got, ref.cpu().numpy()))


def test_noalloc_rejects_sizes_beyond_its_scratch(s1kv, cuda):
    torch = cuda
    L = s1kv.lib()
    pool = s1kv.Pool(1, 8, 128, 64, 16)
    kb, vb = C.c_void_p(), C.c_void_p()
    s1kv.check(L.s1kv_pool_storage(pool.h, 0, C.byref(kb), C.byref(vb)))
    n, max_len = 4096, 1 << 20  # far more partial results than 8 MiB holds
    tables = torch.zeros((n, max_len // 16), dtype=torch.int32, device="cuda")
    lens = torch.ones(n, dtype=torch.int32, device="cuda")
    q = torch.zeros((n, 32, 128), device="cuda")
    out = torch.zeros_like(q)
    st = L.s1kv_decode_attention_noalloc(kb, vb, s1kv.DTYPE_F32, 64 * 16, 8, 128, 16, C.c_void_p(tables.data_ptr()),
                                         max_len // 16, C.c_void_p(lens.data_ptr()), n, max_len,
                                         C.c_void_p(q.data_ptr()), C.c_void_p(out.data_ptr()), 32, None)
    assert st == s1kv.EINVAL
    assert "8 MiB" in L.s1kv_last_error().decode()
