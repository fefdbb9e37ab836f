"""Seeded scenarios of the KV-cache path, shared by make_golden.py (which
runs them through the reference's own CPU code), the oracle tests and the
GPU parity tests.

Inputs are regenerated from numpy seeds; the fixtures hold only outputs,
block tables and the seeds.  Each scenario follows the reference's
self_attention order (src/nn/attention.cpp:293-337): curr_pos =
cache.length(seq); rotate q and k at curr_pos; append k, v; paged
attention of q over the sequence.
"""
from __future__ import annotations

import numpy as np

ROPE_BASE = 1.0e6


def randn(rng, *shape):
    return rng.standard_normal(shape, dtype=np.float32)


def remove_trick_plan(max_blocks, order):
    """Ops that leave a fresh reference pool's free list equal to `order`
    (bottom .. top) using only append/remove, as in
    tests/test_attention.cpp:76-78: take every block with a one-block dummy
    sequence, then remove the dummies so blocks are pushed in `order`.
    Dummy i (allocated i-th) holds block max_blocks - 1 - i."""
    holder = {max_blocks - 1 - i: i for i in range(max_blocks)}
    return [holder[int(b)] for b in order]


DUMMY_BASE = 1 << 40


SCENARIOS = {
    # cfg1 shape (24 layers cut to 2): Hq14/Hkv2/D64, bs16, shuffled free
    # list, prefill then decode one token per step.
    "cfg1_small": dict(layers=2, Hq=14, Hkv=2, D=64, bs=16, max_blocks=24, seed=0, seqs=[0], prefill=[40],
                       steps=3),
    # cfg2 shape: Hq32/Hkv8/D128, three ragged sequences, two decode steps.
    "cfg2_small": dict(layers=1, Hq=32, Hkv=8, D=128, bs=16, max_blocks=20, seed=1, seqs=[5, 6, 7],
                       prefill=[17, 40, 70], steps=2),
    # cfg4 group size (8 query heads per kv head).
    "g8_small": dict(layers=1, Hq=16, Hkv=2, D=128, bs=16, max_blocks=16, seed=3, seqs=[1, 2], prefill=[33, 95],
                     steps=1),
}


# BASELINE-sized scenario, pinned by digests (the reference's outputs are
# too large to commit in full): cfg1 exactly -- 24 layers, Hq14/Hkv2/D64,
# RoPE theta 1e6, fp32, block 16, seed 0, free list shuffled (the remove
# trick), prefill 512 tokens then 64 decode steps.  48 physical blocks
# hold the 576 tokens (36 blocks) with room to scatter.
FULL_SCENARIOS = {
    "cfg1": dict(layers=24, Hq=14, Hkv=2, D=64, bs=16, max_blocks=48, seed=0, seqs=[0], prefill=[512], steps=64),
}


def spec(name):
    return SCENARIOS[name] if name in SCENARIOS else FULL_SCENARIOS[name]


def run_scenario(name, backend):
    """Runs a scenario through `backend` and returns its outputs:
    {"out": [layer][step][seq] -> [1, Hq, D], "tables": {seq: [...]},
     "prefill_out": [layer][seq] -> [P, Hq, D]}.

    backend(pool_args) must provide: new_pools(layers, H, D, max_blocks, bs,
    free_order), rope(x, start_pos), append(layer, seq, k, v),
    attention(layer, seq, q, Hq), length(seq), table(seq)."""
    s = spec(name)
    rng = np.random.default_rng(s["seed"])
    order = rng.permutation(s["max_blocks"]).astype(np.int32)
    backend.new_pools(s["layers"], s["Hkv"], s["D"], s["max_blocks"], s["bs"], order)
    L, Hq, Hkv, D = s["layers"], s["Hq"], s["Hkv"], s["D"]
    res = {"out": [[[None] * len(s["seqs"]) for _ in range(s["steps"])] for _ in range(L)],
           "prefill_out": [[None] * len(s["seqs"]) for _ in range(L)]}
    # prefill: each sequence's whole prompt at once, layer by layer
    for si, (seq, P) in enumerate(zip(s["seqs"], s["prefill"])):
        for layer in range(L):
            q = randn(rng, P, Hq, D)
            k = randn(rng, P, Hkv, D)
            v = randn(rng, P, Hkv, D)
            pos = backend.length(seq, layer)
            qr, kr = backend.rope(q, pos), backend.rope(k, pos)
            backend.append(layer, seq, kr, v)
            res["prefill_out"][layer][si] = backend.attention(layer, seq, qr, Hq)
    for step in range(s["steps"]):
        for si, seq in enumerate(s["seqs"]):
            for layer in range(L):
                q = randn(rng, 1, Hq, D)
                k = randn(rng, 1, Hkv, D)
                v = randn(rng, 1, Hkv, D)
                pos = backend.length(seq, layer)
                qr, kr = backend.rope(q, pos), backend.rope(k, pos)
                backend.append(layer, seq, kr, v)
                res["out"][layer][step][si] = backend.attention(layer, seq, qr, Hq)
    res["tables"] = {seq: np.asarray(backend.table(seq), np.int32) for seq in s["seqs"]}
    return res


def scenario_inputs(name):
    """Regenerates every input of a scenario in the order run_scenario
    draws them: (order, prefill[(layer, seq)] -> (q, k, v),
    decode[(step, seq, layer)] -> (q, k, v))."""
    s = spec(name)
    rng = np.random.default_rng(s["seed"])
    order = rng.permutation(s["max_blocks"]).astype(np.int32)
    L, Hq, Hkv, D = s["layers"], s["Hq"], s["Hkv"], s["D"]
    pre, dec = {}, {}
    for seq, P in zip(s["seqs"], s["prefill"]):
        for layer in range(L):
            pre[(layer, seq)] = (randn(rng, P, Hq, D), randn(rng, P, Hkv, D), randn(rng, P, Hkv, D))
    for step in range(s["steps"]):
        for seq in s["seqs"]:
            for layer in range(L):
                dec[(step, seq, layer)] = (randn(rng, 1, Hq, D), randn(rng, 1, Hkv, D), randn(rng, 1, Hkv, D))
    return order, pre, dec


PREFILL_ROWS_KEPT = 4


def flatten(res, name):
    """Scenario result -> flat dict of arrays for np.savez (the last
    PREFILL_ROWS_KEPT query rows of each prefill, every decode output)."""
    s = spec(name)
    out = {}
    for layer in range(s["layers"]):
        for si, seq in enumerate(s["seqs"]):
            out[f"prefill_l{layer}_s{seq}"] = res["prefill_out"][layer][si][-PREFILL_ROWS_KEPT:]
            for step in range(s["steps"]):
                out[f"dec_l{layer}_t{step}_s{seq}"] = res["out"][layer][step][si]
    for seq, t in res["tables"].items():
        out[f"table_s{seq}"] = t
    return out


def output_keys(name):
    """Keys of every attention output of a scenario: the whole prefill
    output of each (layer, sequence) and each decode output."""
    s = spec(name)
    keys = []
    for layer in range(s["layers"]):
        for seq in s["seqs"]:
            keys.append(f"prefill_l{layer}_s{seq}")
            keys += [f"dec_l{layer}_t{t}_s{seq}" for t in range(s["steps"])]
    return keys


def outputs(res, name):
    """Scenario result -> {output key: array} (every output, full size)."""
    s = spec(name)
    out = {}
    for layer in range(s["layers"]):
        for si, seq in enumerate(s["seqs"]):
            out[f"prefill_l{layer}_s{seq}"] = res["prefill_out"][layer][si]
            for t in range(s["steps"]):
                out[f"dec_l{layer}_t{t}_s{seq}"] = res["out"][layer][t][si]
    return out


def digest(a):
    """SHA-256 of an output's fp32 bytes (C order): bit-exact identity."""
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).digest()


# Outputs a full-size fixture keeps as values (besides every digest): the
# first and last layer at the first, middle and last decode step, and the
# last PREFILL_ROWS_KEPT prefill rows of those layers.
def kept_values(name):
    s = spec(name)
    layers = sorted({0, s["layers"] - 1})
    steps = sorted({0, s["steps"] // 2, s["steps"] - 1})
    return [(f"prefill_l{l}_s{q}", True) for l in layers for q in s["seqs"]] + \
           [(f"dec_l{l}_t{t}_s{q}", False) for l in layers for t in steps for q in s["seqs"]]


# ---------------------------------------------------------------- pool ops --

def pool_ops(seed, n_ops=60, max_blocks=12, bs=4):
    """A seeded random op script for block-pool bookkeeping (H=1, D=2)."""
    rng = np.random.default_rng(seed)
    ops = []
    live = set()
    for _ in range(n_ops):
        r = rng.random()
        seq = int(rng.integers(0, 5))
        if r < 0.55:
            ops.append(("append", seq, int(rng.integers(0, 11))))
            live.add(seq)
        elif r < 0.8:
            ops.append(("truncate", seq, int(rng.integers(0, 14))))
        else:
            ops.append(("remove", seq, 0))
            live.discard(seq)
    return ops
