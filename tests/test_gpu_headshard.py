"""KV-head-sharded decode on two GPUs (one process per GPU, NCCL): each
rank's pool holds half of the KV heads of every token (bf16 storage), runs
the paged decode kernel for the query heads of its groups, and one NCCL
all-gather over NVLink reassembles all heads.  The gathered output is
compared with the oracle's full-head GQA attention on the same bf16-rounded
K/V (tolerance 2e-5 x max |ref|, as for the 1-GPU bf16 path).  Skipped on
a box with fewer than two GPUs."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "s1-infer_b200"))
    import torch
    import torch.distributed as dist

    import s1kv
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    Hq, Hkv, D, bs = 32, 8, 128, 16
    ctx = [300, 517, 1024]
    B = len(ctx)
    rng = np.random.default_rng(7)
    k = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    v = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    q = rng.standard_normal((B, Hq, D), dtype=np.float32)
    kv_lo, kv_hi, q_lo, q_hi = s1kv.head_shard(world, rank, Hkv, Hq)
    need = sum((c + bs - 1) // bs for c in ctx)
    pool = s1kv.Pool(1, kv_hi - kv_lo, D, need + 4, bs, dtype="bf16",
                     initial_free_list=np.random.default_rng(3).permutation(need + 4))
    seqs = list(range(B))
    with pool.batch(seqs, ctx, [0] * B) as b:
        b.append(0, torch.from_numpy(np.concatenate([x[:, kv_lo:kv_hi] for x in k])).cuda().contiguous(),
                 torch.from_numpy(np.concatenate([x[:, kv_lo:kv_hi] for x in v])).cuda().contiguous())
    out_local = pool.attention(0, seqs, [1] * B, torch.from_numpy(q[:, q_lo:q_hi].copy()).cuda(), q_hi - q_lo)
    full = s1kv.gather_heads(out_local, world)
    torch.cuda.synchronize()
    assert pool.check_device() == 0
    pool.close()
    dist.barrier()
    dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), full.cpu().numpy())


@pytest.mark.gpu
def test_two_gpu_head_sharded_decode_matches_oracle(tmp_path, oracle):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank, args=(world, _port(), str(tmp_path)), nprocs=world, start_method="spawn", join=True)
    Hq, Hkv, D = 32, 8, 128
    ctx = [300, 517, 1024]
    rng = np.random.default_rng(7)
    k = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    v = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    q = rng.standard_normal((len(ctx), Hq, D), dtype=np.float32)
    ref = np.stack([oracle.gqa_attention(q[s:s + 1], oracle.bf16_round(k[s]), oracle.bf16_round(v[s]), Hq, Hkv, D)[0]
                    for s in range(len(ctx))])
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert got.shape == ref.shape
        assert np.max(np.abs(got - ref)) <= 2e-5 * np.max(np.abs(ref))


def _rank_fused(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "s1-infer_b200"))
    import torch
    import torch.distributed as dist

    import s1kv
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    Hq, Hkv, D, bs = 32, 8, 128, 16
    ctx = FUSED_CTX
    B = len(ctx)
    rng = np.random.default_rng(7)
    k = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    v = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    qs = rng.standard_normal((3, B, Hq, D), dtype=np.float32)
    kv_lo, kv_hi, q_lo, q_hi = s1kv.head_shard(world, rank, Hkv, Hq)
    need = sum((c + bs - 1) // bs for c in ctx)
    pool = s1kv.Pool(1, kv_hi - kv_lo, D, need + 4, bs, dtype="bf16",
                     initial_free_list=np.random.default_rng(3).permutation(need + 4))
    seqs = list(range(B))
    with pool.batch(seqs, ctx, [0] * B) as b:
        b.append(0, torch.from_numpy(np.concatenate([x[:, kv_lo:kv_hi] for x in k])).cuda().contiguous(),
                 torch.from_numpy(np.concatenate([x[:, kv_lo:kv_hi] for x in v])).cuda().contiguous())
    ex = s1kv.PeerExchange(rank, world, B, Hq, D)
    outs, slices = [], []
    hq = q_hi - q_lo
    with pool.batch(seqs, [0] * B, [1] * B) as b:
        for e in (1, 2, 3):  # both slots, and one reused
            ex.attention(b, 0, torch.from_numpy(qs[e - 1][:, q_lo:q_hi].copy()).cuda(), q_lo, e)
            if e == 2:
                ex.wait(e)
            else:  # the wait fused with a copy of the other rank's heads
                slices.append(ex.wait_copy(e, (1 - rank) * hq, hq, torch.empty((B, hq, D), device="cuda")))
            outs.append(ex.output(e).clone())
    torch.cuda.synchronize()
    assert pool.check_device() == 0
    dist.barrier()  # no rank frees its buffer while a peer may still hold it open
    ex.close()
    pool.close()
    dist.barrier()
    dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"fused{rank}.npy"), torch.stack(outs).cpu().numpy())
    np.save(os.path.join(out_dir, f"slices{rank}.npy"), torch.stack(slices).cpu().numpy())


FUSED_CTX = [300, 517, 1024, 40000]  # the long row: 63 splits, merged in two levels


@pytest.mark.gpu
def test_two_gpu_fused_exchange_matches_oracle(tmp_path, oracle):
    """The decode kernels of each rank store their heads' rows into both
    ranks' token-major buffers over NVLink (no NCCL, no reorder), also the
    rows merged in two levels: three epochs in a row, each rank's buffer
    equals the oracle's full-head attention (2e-5 x max |ref|), and the
    waits fused with a copy of the other rank's heads copy them exactly."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_fused, args=(world, _port(), str(tmp_path)), nprocs=world, start_method="spawn", join=True)
    Hq, Hkv, D = 32, 8, 128
    ctx = FUSED_CTX
    rng = np.random.default_rng(7)
    k = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    v = [rng.standard_normal((c, Hkv, D), dtype=np.float32) for c in ctx]
    qs = rng.standard_normal((3, len(ctx), Hq, D), dtype=np.float32)
    hq = Hq // world
    for r in range(world):
        got = np.load(tmp_path / f"fused{r}.npy")
        sl = np.load(tmp_path / f"slices{r}.npy")
        for e in range(3):
            ref = np.stack([oracle.gqa_attention(qs[e][s:s + 1], oracle.bf16_round(k[s]), oracle.bf16_round(v[s]), Hq,
                                                 Hkv, D)[0] for s in range(len(ctx))])
            assert np.max(np.abs(got[e] - ref)) <= 2e-5 * np.max(np.abs(ref))
        h0 = (1 - r) * hq
        for i, e in enumerate((0, 2)):  # epochs 1 and 3 copied a head range
            np.testing.assert_array_equal(sl[i], got[e][:, h0:h0 + hq])


@pytest.mark.gpu
def test_exchange_wait_times_out_on_an_epoch_nobody_wrote(cuda):
    """A one-rank exchange waiting for an epoch no kernel wrote: the bounded
    wait gives up (about a second), the device error word reports the
    timeout, and the GPU keeps working."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "s1-infer_b200"))
    import s1kv
    ex = s1kv.PeerExchange(0, 1, 2, 8, 64)
    ex.wait(7, force=True)
    torch.cuda.synchronize()
    with pytest.raises(s1kv.S1KVError) as e:
        s1kv.device_check(torch.cuda.current_device())
    assert e.value.status == s1kv.ETIMEOUT
    assert s1kv.device_check(torch.cuda.current_device()) == 0  # read and cleared
    x = torch.ones(4, device="cuda") * 2
    assert float(x.sum()) == 8.0
    ex.close()
