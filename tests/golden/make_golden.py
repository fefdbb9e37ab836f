"""Generates the golden fixtures in this directory by running the
reference's own CPU implementation (oracle/_ref/libs1ref.so, compiled from
the reference sources by oracle/Makefile).

    python tests/golden/make_golden.py

Writes:
  rope.npz        apply_rope outputs (src/nn/RoPE.cpp) for seeded inputs
  pool_ops.npz    KVBlockPool bookkeeping (status, length, block table)
                  after every op of seeded op scripts
  int8.npz        quantize_tensor / matmul_quantized outputs
                  (src/quantized_tensor.cpp) on the inputs of the reference's
                  tests/test_quantized_tensor.cpp and on seeded matrices
  <scenario>.npz  paged-attention outputs and block tables of the scenarios
                  in scenarios.py (prefill + decode through KVBlockPool,
                  apply_rope, GQA_attention_paged)
  cfg1_full.npz   the same for the full cfg1 workload (24 layers, prefill
                  512, 64 decode steps): SHA-256 of every output, a few
                  outputs as values, the block table

  logits.npz      final logits of the reference's own model code over a
                  seeded random-weight Qwen3-0.6B-shaped model
                  (tests/cpp/logits_parity.cpp): argmax, SHA-256 and the 32
                  largest logits of each of 8 cached decode steps

    python tests/golden/make_golden.py [--only-full | --only-logits]
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from oracle import oracle as O  # noqa: E402
import scenarios as S  # noqa: E402


class RefBackend:
    """One reference KVBlockPool per layer, as src/demo.cpp:56-59 builds."""

    def new_pools(self, layers, H, D, max_blocks, bs, order):
        self.pools = [O.RefPool(H, D, max_blocks, bs) for _ in range(layers)]
        self.bs = bs
        plan = S.remove_trick_plan(max_blocks, order)
        for p in self.pools:
            z = np.zeros((bs, H, D), np.float32)
            for i in range(max_blocks):
                assert p.append(S.DUMMY_BASE + i, z, z) == 0
            for i in plan:
                assert p.remove(S.DUMMY_BASE + i) == 0

    def rope(self, x, pos):
        return O.ref_apply_rope(x, pos)

    def append(self, layer, seq, k, v):
        assert self.pools[layer].append(seq, k, v) == 0

    def attention(self, layer, seq, q, Hq):
        return self.pools[layer].attention(seq, q, Hq)

    def length(self, seq, layer=0):
        return self.pools[layer].length(seq)

    def table(self, seq):
        tabs = [p.block_table(seq) for p in self.pools]
        for t in tabs[1:]:
            assert np.array_equal(t, tabs[0]), "per-layer tables must agree"
        return tabs[0]


def make_rope():
    out = {}
    rng = np.random.default_rng(11)
    for D in (4, 64, 128):
        x = rng.standard_normal((3, 2, D), dtype=np.float32)
        out[f"x_{D}"] = x
        for pos in (0, 1, 4095, 131071):
            out[f"out_{D}_{pos}"] = O.ref_apply_rope(x, pos)
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **out)


def make_pool_ops():
    out = {}
    for seed in range(4):
        ops = S.pool_ops(seed)
        p = O.RefPool(1, 2, 12, 4)
        rng = np.random.default_rng(100 + seed)
        status, lengths, tables = [], [], []
        for kind, seq, n in ops:
            if kind == "append":
                k = rng.standard_normal((n, 1, 2), dtype=np.float32)
                st = p.append(seq, k, k)
            elif kind == "truncate":
                st = p.truncate(seq, n)
            else:
                st = p.remove(seq)
            status.append(st)
            lengths.append(p.length(seq))
            t = p.block_table(seq)
            tables.append(-np.ones(12, np.int32) if t is None else np.pad(t, (0, 12 - len(t)), constant_values=-2))
        out[f"ops_{seed}"] = np.array([[["append", "truncate", "remove"].index(k), s, n] for k, s, n in ops], np.int64)
        out[f"status_{seed}"] = np.array(status, np.int32)
        out[f"length_{seed}"] = np.array(lengths, np.int64)
        out[f"tables_{seed}"] = np.stack(tables)
    np.savez_compressed(os.path.join(HERE, "pool_ops.npz"), **out)


def int8_cases():
    """(name, w [K, N], x [M, K]) inputs of the int8 fixtures."""
    cases = []
    # tests/test_quantized_tensor.cpp:5-23, 26-39, 42-49
    cases.append(("kat_2x3", np.array([[1.0, -2.0, 0.5], [10.0, -20.0, 5.0]], np.float32),
                  np.array([[0.5, -1.0]], np.float32)))
    cases.append(("kat_per_row", np.array([[0.01, 0.02], [1.0, 2.0]], np.float32), np.array([[1.0, 1.0]], np.float32)))
    cases.append(("kat_zero_row", np.zeros((1, 2), np.float32), np.array([[3.0]], np.float32)))
    # tests/test_quantized_tensor.cpp:51-75: M 2, K 80, N 88.  The index
    # expressions are size_t: (i * 13) % 200 - 100 wraps below zero to about
    # 2^64, which becomes 1.8446744e19f before the 0.01f scale.
    def ref_fill(n, mul):
        i = np.arange(n, dtype=np.uint64)
        v = ((i * np.uint64(mul)) % np.uint64(200)) - np.uint64(100)  # wraps like size_t
        return (np.float32(0.01) * v.astype(np.float32)).astype(np.float32)
    cases.append(("kat_blocked", ref_fill(80 * 88, 7).reshape(80, 88), ref_fill(2 * 80, 13).reshape(2, 80)))
    rng = np.random.default_rng(11)
    for name, (M, K, N) in {"rand_1x384x136": (1, 384, 136), "rand_3x257x131": (3, 257, 131),
                            "rand_9x200x72": (9, 200, 72)}.items():
        w = (rng.standard_normal((K, N)) * rng.uniform(0.01, 2.0, size=(K, 1))).astype(np.float32)
        w[5] = 0.0  # an all-zero row
        cases.append((name, w, rng.standard_normal((M, K)).astype(np.float32)))
    return cases


def make_int8():
    out = {}
    for name, w, x in int8_cases():
        q, sc = O.ref_quantize_rows(w)
        out[f"{name}/w"], out[f"{name}/x"] = w, x
        out[f"{name}/q"], out[f"{name}/scales"] = q, sc
        out[f"{name}/out"] = O.ref_matmul_int8(x, q, sc)
        assert np.array_equal(out[f"{name}/out"].view(np.uint32), O.ref_matmul_int8(x, q, sc, threaded=True).view(np.uint32))
    np.savez_compressed(os.path.join(HERE, "int8.npz"), **out)


def make_full(name):
    """A BASELINE-sized scenario (scenarios.FULL_SCENARIOS): the SHA-256 of
    every attention output of the reference (pins the oracle bit for bit at
    full size), a few outputs as values, and the block tables."""
    res = S.run_scenario(name, RefBackend())
    outs = S.outputs(res, name)
    keys = S.output_keys(name)
    fx = {"keys": np.array(keys), "sha256": np.stack([np.frombuffer(S.digest(outs[k]), np.uint8) for k in keys])}
    for key, prefill in S.kept_values(name):
        fx["value/" + key] = outs[key][-S.PREFILL_ROWS_KEPT:] if prefill else outs[key]
    for seq, t in res["tables"].items():
        fx[f"table_s{seq}"] = t
    np.savez_compressed(os.path.join(HERE, f"{name}_full.npz"), **fx)


LOGITS_ARGS = {"prompt": 64, "steps": 8, "vocab": 151936, "seed": 1}


def read_logits(path):
    """(argmax [steps], logits [steps, vocab]) of a logits_parity output."""
    raw = np.fromfile(path, np.int32)
    steps, vocab = int(raw[0]), int(raw[1])
    rec = raw[2:].reshape(steps, 1 + vocab)
    return rec[:, 0].copy(), rec[:, 1:].copy().view(np.float32)


def make_logits():
    """The reference's final logits over the seeded random-weight model
    (oracle/_ref/logits_ref, tests/cpp/logits_parity.cpp) in both modes:
    per step the argmax, the SHA-256 of the logits and the 32 largest."""
    import hashlib
    import subprocess
    import tempfile
    exe = os.path.join(ROOT, "oracle", "_ref", "logits_ref")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "logits"], check=True)
    a = LOGITS_ARGS
    out = {k: np.int64(v) for k, v in a.items()}
    for mode in ("f32", "int8"):
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "l.bin")
            subprocess.run([exe, mode, str(a["prompt"]), str(a["steps"]), str(a["vocab"]), str(a["seed"]), path],
                           check=True, capture_output=True)
            am, lg = read_logits(path)
        top = np.argsort(-lg, axis=1, kind="stable")[:, :32]
        out[f"{mode}/argmax"] = am
        out[f"{mode}/sha256"] = np.stack([np.frombuffer(hashlib.sha256(r.tobytes()).digest(), np.uint8) for r in lg])
        out[f"{mode}/top_idx"] = top.astype(np.int32)
        out[f"{mode}/top_val"] = np.take_along_axis(lg, top, axis=1)
    np.savez_compressed(os.path.join(HERE, "logits.npz"), **out)


def main():
    O.build()
    if not O.ref_available():
        sys.exit("oracle/_ref/libs1ref.so missing: the reference sources are needed to make fixtures")
    if "--only-full" in sys.argv:
        for name in S.FULL_SCENARIOS:
            make_full(name)
        return
    if "--only-logits" in sys.argv:
        make_logits()
        return
    make_rope()
    make_pool_ops()
    make_int8()
    for name in S.SCENARIOS:
        res = S.run_scenario(name, RefBackend())
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **S.flatten(res, name))
    for name in S.FULL_SCENARIOS:
        make_full(name)
    make_logits()
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
