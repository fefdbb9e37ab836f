"""Pool churn (continuous batching with prefix reuse and LRU eviction) on
the host: the request stream's statistics, and the step driver's
bookkeeping on a host-only pool, replayed on the oracle pool and compared
bit for bit (free list, LRU order, block tables, refcounts)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def test_workload_statistics(s1kv):
    from s1kv.churn import ChurnWorkload
    wl = ChurnWorkload(seed=4)
    reqs = [wl.request() for _ in range(20000)]
    lens = np.array([len(t) for t, _ in reqs])
    outs = np.array([o for _, o in reqs])
    assert abs(np.median(lens) / 1024 - 1) < 0.05
    assert abs(lens.mean() / 1410 - 1) < 0.05  # exp(mu + sigma^2 / 2) = 1024 * e^0.32
    assert outs.min() >= 32 and outs.max() <= 512
    assert len(wl.prefixes) == 16 and all(256 <= len(p) <= 4096 for p in wl.prefixes)
    reused = sum(any(np.array_equal(t[:min(64, len(t))], p[:min(64, len(t))]) for p in wl.prefixes) for t, _ in reqs)
    assert abs(reused / len(reqs) - 0.3) < 0.02
    assert abs(np.mean([wl.arrivals() for _ in range(20000)]) - 1.0) < 0.03


def _run(s1kv, steps, max_blocks, seed=9):
    from churn_replay import HostBatchPool
    from s1kv.churn import ChurnDriver, ChurnWorkload
    order = np.random.default_rng(seed).permutation(max_blocks).astype(np.int32)
    pool = HostBatchPool(s1kv.Pool(1, 1, 8, max_blocks, 16, host_only=True, initial_free_list=order))
    wl = ChurnWorkload(seed=seed, arrival_rate=1.5, prefix_len=(32, 512), prompt_median=96, out_len=(8, 64),
                       max_prompt=1024)
    drv = ChurnDriver(pool, wl, max_running=24, headroom=4)
    drv.queue.extend(wl.request() for _ in range(24))
    for _ in range(steps):
        plan = drv.plan()
        with drv.open(plan):
            pass
        drv.close(plan)
    return pool, drv, order


def test_churn_bookkeeping_matches_oracle(s1kv, oracle):
    from churn_replay import replay
    max_blocks = 600
    pool, drv, order = _run(s1kv, 600, max_blocks)
    st = pool.stats()
    assert drv.stats["retired"] > 50 and drv.stats["admitted"] > 50
    assert st["evictions"] > 0 and drv.stats["prefix_hit_tokens"] > 0
    opool = oracle.Pool(1, 8, max_blocks, 16, free_order=order)
    replay(drv.log, opool)
    assert np.array_equal(pool.free_list(), opool.free_list())
    assert np.array_equal(pool.lru_list(), opool.lru_list())
    assert np.array_equal(pool.refcounts(), opool.refcounts())
    for s in drv.running:
        assert np.array_equal(pool.block_table(s), opool.block_table(s))
        assert pool.length(s) == opool.length(s)
    # every block is free, cached in the LRU, or referenced
    rc = pool.refcounts()
    assert st["num_free"] + st["num_lru"] + int((rc > 0).sum()) == max_blocks


def test_churn_defers_and_preempts_when_the_pool_is_full(s1kv, oracle):
    from churn_replay import replay
    max_blocks = 160  # far too small for 24 running sequences
    pool, drv, order = _run(s1kv, 300, max_blocks, seed=5)
    assert drv.stats["deferred"] + drv.stats["preempted"] > 0
    opool = oracle.Pool(1, 8, max_blocks, 16, free_order=order)
    replay(drv.log, opool)
    assert np.array_equal(pool.free_list(), opool.free_list())
    assert np.array_equal(pool.lru_list(), opool.lru_list())
    for s in drv.running:
        assert np.array_equal(pool.block_table(s), opool.block_table(s))
