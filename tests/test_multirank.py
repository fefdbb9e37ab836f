"""Multi-GPU logic on CPU: the sequence-sharded path the bench runs under
torchrun (one process and one independent pool per GPU, no collective on
the data path), exercised with world_size 2 over gloo.  Each rank builds a
host-only pool for its share of the global batch, places every sequence's
blocks, and the ranks reduce their numbers with the bench's own
max/sum helpers."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_every_rank_gets_the_one_gpu_workload(n):
    sys.path.insert(0, ROOT)
    import bench
    shares = bench.contexts(n)
    assert len(shares) == n and all(s == shares[0] for s in shares)
    assert len(shares[0]) == bench.SEQS_PER_GPU
    assert all(bench.CTX_LO <= c <= bench.CTX_HI for c in shares[0])


@pytest.mark.parametrize("n", [2, 4, 8])
def test_balanced_shards_cover_a_shared_batch(n):
    sys.path.insert(0, ROOT)
    import bench
    ctx = list(np.random.default_rng(3).integers(128, 4097, size=64 * n))
    shares = bench.balanced_shards(ctx, n)
    assert sorted(sum(shares, [])) == sorted(int(c) for c in ctx)
    loads = [sum(s) for s in shares]
    assert max(loads) / min(loads) < 1.01


def _rank_main(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "s1-infer_b200"))
    import torch
    import torch.distributed as dist

    import bench
    import s1kv
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    share = bench.contexts(world)[rank]
    need = sum((c + bench.BS - 1) // bench.BS for c in share)
    pool = s1kv.Pool(bench.LAYERS, bench.HKV, bench.D, int(need * 1.25), bench.BS, host_only=True,
                     initial_free_list=np.random.default_rng(1000 + rank).permutation(int(need * 1.25)))
    for s, c in enumerate(share):
        st, slots = pool.reserve(s, c)
        assert st == 0 and len(slots) == c
    used = int(need * 1.25) - len(pool.free_list())
    tokens = bench.sum_over_ranks(torch, world, float(sum(share)))
    slowest = bench.max_over_ranks(torch, world, float(rank + 1))
    gathered = [None] * world
    dist.all_gather_object(gathered, bench.balanced_shards(sum(bench.contexts(world), []), world)[rank])
    dist.barrier()
    dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"),
            np.array([used, need, tokens, slowest, len(sum(gathered, []))], np.float64))


def test_two_rank_gloo_sharded_pools(tmp_path):
    import torch.multiprocessing as mp
    world, port = 2, free_port()
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn", join=True)
    import bench
    shares = bench.contexts(world)
    for r in range(world):
        used, need, tokens, slowest, n_all = np.load(tmp_path / f"rank{r}.npy")
        assert used == need  # every block of the share placed, none shared
        assert tokens == sum(sum(s) for s in shares)
        assert slowest == world
        assert n_all == world * bench.SEQS_PER_GPU


def _head_rank_main(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "s1-infer_b200"))
    import torch
    import torch.distributed as dist

    import s1kv
    from oracle import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    Hq, Hkv, D, B = 16, 4, 64, 3
    rng = np.random.default_rng(11)
    ctx = [37, 90, 64]
    k = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    v = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    q = rng.standard_normal((B, Hq, D), dtype=np.float32)
    kv_lo, kv_hi, q_lo, q_hi = s1kv.head_shard(world, rank, Hkv, Hq)
    # this rank's share: its KV heads and the query heads of their groups
    local = np.stack([oracle.gqa_attention(q[s:s + 1, q_lo:q_hi], k[s][:, kv_lo:kv_hi], v[s][:, kv_lo:kv_hi],
                                           q_hi - q_lo, kv_hi - kv_lo, D)[0] for s in range(B)])
    full = s1kv.gather_heads(torch.from_numpy(local), world).numpy()
    ref = np.stack([oracle.gqa_attention(q[s:s + 1], k[s], v[s], Hq, Hkv, D)[0] for s in range(B)])
    dist.barrier()
    dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"head{rank}.npy"), np.stack([full, ref]))


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_gather_reassembles_full_attention(tmp_path, world):
    """KV-head sharding: each gloo rank computes the attention of its own KV
    heads' groups; the all-gather and head-major to token-major reorder give
    every rank exactly the full-head result."""
    import torch.multiprocessing as mp
    mp.start_processes(_head_rank_main, args=(world, free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    for r in range(world):
        full, ref = np.load(tmp_path / f"head{r}.npy")
        assert np.array_equal(full, ref)


def test_head_shard_partition():
    sys.path.insert(0, os.path.join(ROOT, "s1-infer_b200"))
    import s1kv
    for world in (1, 2, 4, 8):
        parts = [s1kv.head_shard(world, r, 8, 64) for r in range(world)]
        assert [p[0] for p in parts] == list(range(0, 8, 8 // world))
        assert parts[-1][1] == 8 and parts[-1][3] == 64
        for kv_lo, kv_hi, q_lo, q_hi in parts:  # whole GQA groups
            assert q_lo == kv_lo * 8 and q_hi == kv_hi * 8
    with pytest.raises(ValueError):
        s1kv.head_shard(3, 0, 8, 64)
