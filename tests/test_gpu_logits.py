"""Final-logits parity through the reference's own model code.

tests/cpp/logits_parity.cpp builds a seeded random-weight model of the
reference's shape (Qwen3-0.6B: 28 layers, hidden 1024, 16/8 heads of 128,
MLP 3072, vocabulary 151,936) and runs the 8-step cached greedy decode of
tests/test_kv_cache_correctness.cpp:28-114 (prompt of 64 seeded token ids,
then one token per step) through model_forward (f32) and
model_forward_quantized (int8).  oracle/Makefile links it twice from the
reference's sources: logits_ref with the reference's own KV path on the CPU
(the oracle), logits_on_shim with KVBlockPool, apply_rope, GQA_attention,
GQA_attention_paged and the int8 matmul from the B200 engine (the drop-in).

Checked per step: the oracle's logits equal the fixture made from the same
program in another container bit for bit (SHA-256), the argmax tokens are
equal, and max |shim - ref| <= 2e-5 x max |ref| over the whole vocabulary
(the north-star fp32 bound for final logits).  The engine must have
launched its kernels (the GQA functions of src/nn/attention.cpp are
shadowed, not used)."""
import hashlib
import os
import re
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF_DIR = os.path.join(ROOT, "oracle", "_ref")
sys.path.insert(0, os.path.join(HERE, "golden"))

pytestmark = pytest.mark.gpu

TOL = 2e-5


def read_logits(path):
    raw = np.fromfile(path, np.int32)
    steps, vocab = int(raw[0]), int(raw[1])
    rec = raw[2:].reshape(steps, 1 + vocab)
    return rec[:, 0].copy(), rec[:, 1:].copy().view(np.float32)


@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_final_logits_match_reference_model(cuda, tmp_path, mode):
    g = np.load(os.path.join(HERE, "golden", "logits.npz"))
    args = [str(int(g[k])) for k in ("prompt", "steps", "vocab", "seed")]
    exes = {name: os.path.join(REF_DIR, name) for name in ("logits_ref", "logits_on_shim")}
    for e in exes.values():
        assert os.path.exists(e), f"{e} missing: build with `make -C oracle logits` where the reference sources are"
    procs = {name: subprocess.Popen([e, mode, *args, str(tmp_path / f"{name}.bin")], stdout=subprocess.PIPE,
                                    stderr=subprocess.STDOUT, text=True) for name, e in exes.items()}
    logs = {name: p.communicate(timeout=1200)[0] for name, p in procs.items()}
    for name, p in procs.items():
        assert p.returncode == 0, (name, logs[name][-2000:])
    am_ref, ref = read_logits(tmp_path / "logits_ref.bin")
    am, got = read_logits(tmp_path / "logits_on_shim.bin")
    for i in range(ref.shape[0]):
        assert hashlib.sha256(ref[i].tobytes()).digest() == g[f"{mode}/sha256"][i].tobytes(), f"oracle step {i}"
    np.testing.assert_array_equal(am_ref, g[f"{mode}/argmax"])
    np.testing.assert_array_equal(am, am_ref)
    errs = np.abs(got.astype(np.float64) - ref).max(axis=1) / np.abs(ref).max(axis=1)
    launches = int(re.search(r"engine launches (\d+)", logs["logits_on_shim"]).group(1))
    print(f"final logits ({mode}): 8 steps x {ref.shape[1]} logits, argmax equal, rel max-abs err per step "
          + " ".join(f"{e:.1e}" for e in errs) + f"; {launches} engine kernel launches")
    assert launches > 0
    assert errs.max() <= TOL, errs
