"""Pool churn on the GPU: the continuous-batching driver runs the real
batch path (all-or-nothing reservation with LRU eviction, RoPE + append of
prompts and decode tokens, paged decode attention on bf16 storage) for 120
steps on a pool small enough to evict.  Then: the bookkeeping equals the
oracle pool's replay of the same operations bit for bit; K read through
the device block tables equals the storage rows the host tables name (the
device mirror is current, including copy-on-write tails and reused evicted
blocks); decode attention over every running sequence matches the oracle
on the same bf16 K/V (2e-5 x max |ref|)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "tests"))


@pytest.mark.gpu
def test_churn_on_device_matches_oracle(s1kv, oracle, cuda):
    import torch
    from churn_replay import replay
    from s1kv.churn import ChurnDriver, ChurnWorkload
    L, Hkv, Hq, D, bs, max_blocks = 2, 2, 8, 128, 16, 700
    order = np.random.default_rng(21).permutation(max_blocks).astype(np.int32)
    pool = s1kv.Pool(L, Hkv, D, max_blocks, bs, dtype="bf16", initial_free_list=order, max_seqs=64)
    wl = ChurnWorkload(seed=21, arrival_rate=1.5, prefix_len=(32, 512), prompt_median=96, out_len=(8, 64),
                       max_prompt=1024)
    drv = ChurnDriver(pool, wl, max_running=24, headroom=4)
    drv.queue.extend(wl.request() for _ in range(24))
    gen = torch.Generator(device="cuda").manual_seed(5)
    for _ in range(120):
        plan = drv.plan()
        with drv.open(plan) as b:
            for layer in range(L):
                k = torch.randn((plan.n_tokens, Hkv, D), device="cuda", generator=gen)
                v = torch.randn((plan.n_tokens, Hkv, D), device="cuda", generator=gen)
                q = torch.randn((plan.n_rows, Hq, D), device="cuda", generator=gen) if plan.n_rows else None
                qr = b.rope_append(layer, k, v, q=q)
                if plan.n_rows:
                    b.attention(layer, qr)
        drv.close(plan)
    torch.cuda.synchronize()
    assert pool.check_device() == 0
    st = pool.stats()
    assert st["evictions"] > 0 and drv.stats["retired"] > 10 and drv.stats["prefix_hit_tokens"] > 0

    opool = oracle.Pool(Hkv, D, max_blocks, bs, free_order=order)
    replay(drv.log, opool)
    assert np.array_equal(pool.free_list(), opool.free_list())
    assert np.array_equal(pool.lru_list(), opool.lru_list())
    seqs = list(drv.running)
    for s in seqs:
        assert np.array_equal(pool.block_table(s), opool.block_table(s))

    kst = pool.read_storage(0, 0)  # bf16 bits, [slots, Hkv, D]
    q = np.random.default_rng(3).standard_normal((len(seqs), Hq, D)).astype(np.float32)
    out = pool.attention(0, seqs, [1] * len(seqs), torch.from_numpy(q).cuda(), Hq).cpu().numpy()
    for i, s in enumerate(seqs):
        n = pool.length(s)
        tab = pool.block_table(s)
        slots = np.array([tab[t // bs] * bs + t % bs for t in range(n)])
        kg = pool.gather(0, s, 0).cpu().numpy()
        assert np.array_equal(kg.view(np.uint32) >> 16, kst[slots].astype(np.uint32))
        vg = pool.gather(0, s, 1).cpu().numpy()
        ref = oracle.gqa_attention(q[i:i + 1], kg, vg, Hq, Hkv, D)
        assert np.max(np.abs(out[i] - ref[0])) <= 2e-5 * np.max(np.abs(ref))
    pool.close()


@pytest.mark.gpu
def test_mixed_step_rotates_each_query_row_at_its_position(s1kv, oracle, cuda):
    """One batch appends a prompt without queries (q_len 0) next to decode
    rows: q is rotated per row at the row's own position (bit-exact with the
    oracle's RoPE), and the appended K bytes are the rotated keys."""
    import torch
    Hkv, Hq, D, bs = 2, 4, 64, 16
    pool = s1kv.Pool(1, Hkv, D, 64, bs)
    rng = np.random.default_rng(12)
    lens0 = {1: 10, 2: 33}
    with pool.batch([1, 2], [10, 33], [0, 0]) as b:
        b.rope_append(0, torch.from_numpy(rng.standard_normal((43, Hkv, D), dtype=np.float32)).cuda(),
                      torch.from_numpy(rng.standard_normal((43, Hkv, D), dtype=np.float32)).cuda())
    # step: seq 3 appends a 7-token prompt (no query rows); seqs 1, 2 decode one token
    k = rng.standard_normal((9, Hkv, D), dtype=np.float32)
    q = rng.standard_normal((2, Hq, D), dtype=np.float32)
    with pool.batch([1, 2, 3], [1, 1, 7], [1, 1, 0]) as b:
        qr = b.rope_append(0, torch.from_numpy(k).cuda(), torch.from_numpy(k).cuda(),
                           q=torch.from_numpy(q).cuda()).cpu().numpy()
    for r, s in enumerate((1, 2)):
        ref = oracle.apply_rope(q[r:r + 1], pos=np.array([lens0[s]]))
        assert np.array_equal(qr[r:r + 1], ref)
    kst = pool.read_storage(0, 0)
    tab = pool.block_table(3)
    slots = [tab[t // bs] * bs + t % bs for t in range(7)]
    assert np.array_equal(kst[slots], oracle.apply_rope(k[2:], pos=np.arange(7)))
    assert pool.check_device() == 0
    pool.close()
