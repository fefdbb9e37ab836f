"""s1kv_batch_layer_host (host buffers, copies overlapped with the kernels
of neighbouring calls on the pool's copy streams) against the same step on
device buffers: appended K/V bytes and attention outputs identical, for a
step of several layers, outputs read after the batch ends."""
import numpy as np
import pytest


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_layer_host_matches_device_path(s1kv, cuda, dtype):
    torch = cuda
    rng = np.random.default_rng(7)
    L, Hq, Hkv, D, bs = 5, 32, 8, 128, 16
    ctx = [37, 300, 129, 1000]
    seqs = [1, 2, 3, 4]
    pools = [s1kv.Pool(L, Hkv, D, 256, bs, dtype=dtype) for _ in range(2)]
    for pool in pools:  # same prompts in both pools
        k = torch.from_numpy(rng.standard_normal((sum(ctx), Hkv, D), dtype=np.float32)).cuda()
        with pool.batch(seqs, ctx, [0] * len(ctx)) as b:
            for layer in range(L):
                b.rope_append(layer, k, k)
        rng = np.random.default_rng(7)
    B = len(seqs)
    q = rng.standard_normal((L, B, Hq, D), dtype=np.float32)
    kn = rng.standard_normal((L, B, Hkv, D), dtype=np.float32)
    vn = rng.standard_normal((L, B, Hkv, D), dtype=np.float32)
    # device path
    dev_out = []
    with pools[0].batch(seqs, [1] * B) as b:
        for layer in range(L):
            qr = b.rope_append(layer, torch.from_numpy(kn[layer]).cuda(), torch.from_numpy(vn[layer]).cuda(),
                               q=torch.from_numpy(q[layer]).cuda())
            dev_out.append(b.attention(layer, qr).cpu().numpy())
    # host path: pinned buffers, every layer's output written asynchronously
    hq, hk, hv = (torch.from_numpy(a).pin_memory() for a in (q, kn, vn))
    ho = torch.full((L, B, Hq, D), float("nan")).pin_memory()
    with pools[1].batch(seqs, [1] * B) as b:
        for layer in range(L):
            b.layer_host(layer, hq[layer], hk[layer], hv[layer], ho[layer], Hq)
    torch.cuda.synchronize()
    for layer in range(L):
        assert np.array_equal(ho[layer].numpy().view(np.uint32), dev_out[layer].view(np.uint32)), layer
        for which in (0, 1):
            assert np.array_equal(pools[0].read_storage(layer, which), pools[1].read_storage(layer, which))
    for pool in pools:
        assert pool.check_device() == 0
        pool.close()


@pytest.mark.gpu
def test_layer_host_batches_of_different_sizes(s1kv, cuda):
    # the copy slots move when a batch's sizes change; a batch must not write
    # memory that the previous batch's copies or kernels still use
    torch = cuda
    L, Hq, Hkv, D, bs = 3, 32, 8, 128, 16
    rng = np.random.default_rng(11)
    pools = [s1kv.Pool(L, Hkv, D, 256, bs) for _ in range(2)]
    ctx = [200, 64, 513, 90]
    k0 = rng.standard_normal((sum(ctx), Hkv, D), dtype=np.float32)
    for pool in pools:
        with pool.batch([1, 2, 3, 4], ctx, [0] * 4) as b:
            for layer in range(L):
                b.rope_append(layer, torch.from_numpy(k0).cuda(), torch.from_numpy(k0).cuda())
    for seqs in ([1, 2, 3, 4], [2, 4], [1, 2, 3, 4]):
        B = len(seqs)
        q = rng.standard_normal((L, B, Hq, D), dtype=np.float32)
        kn = rng.standard_normal((L, B, Hkv, D), dtype=np.float32)
        dev_out = []
        with pools[0].batch(seqs, [1] * B) as b:
            for layer in range(L):
                qr = b.rope_append(layer, torch.from_numpy(kn[layer]).cuda(), torch.from_numpy(kn[layer]).cuda(),
                                   q=torch.from_numpy(q[layer]).cuda())
                dev_out.append(b.attention(layer, qr).cpu().numpy())
        hq, hk = torch.from_numpy(q).pin_memory(), torch.from_numpy(kn).pin_memory()
        ho = torch.full((L, B, Hq, D), float("nan")).pin_memory()
        with pools[1].batch(seqs, [1] * B) as b:
            for layer in range(L):
                b.layer_host(layer, hq[layer], hk[layer], hk[layer], ho[layer], Hq)
        torch.cuda.synchronize()
        for layer in range(L):
            assert np.array_equal(ho[layer].numpy().view(np.uint32), dev_out[layer].view(np.uint32)), (seqs, layer)
    for pool in pools:
        assert pool.check_device() == 0
        pool.close()
