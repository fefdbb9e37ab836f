"""The C++ shim with the reference's interface (s1-infer_b200/shim).

CPU: the shim library exports the reference's C++ entry points with the
reference's signatures.  GPU: the shim's own test program and the
reference's unit tests (tests/test_kv_block_pool.cpp, test_attention.cpp,
test_rope.cpp, compiled unchanged against the shim by
`make -C oracle shimtests`) pass on the device."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM_LIB = os.path.join(ROOT, "s1-infer_b200", "lib", "libs1kv_shim.so")
REF_DIR = os.path.join(ROOT, "oracle", "_ref")

EXPECTED = [
    "KVBlockPool::KVBlockPool(unsigned long, unsigned long, unsigned long, unsigned long)",
    "KVBlockPool::append(unsigned long, std::shared_ptr<Tensor> const&, std::shared_ptr<Tensor> const&)",
    "KVBlockPool::get_k(unsigned long) const",
    "KVBlockPool::get_v(unsigned long) const",
    "KVBlockPool::length(unsigned long) const",
    "KVBlockPool::remove(unsigned long)",
    "KVBlockPool::truncate(unsigned long, unsigned long)",
    "KVBlockPool::get_k_view(unsigned long) const",
    "KVBlockPool::get_v_view(unsigned long) const",
    "GQA_attention_paged(std::shared_ptr<Tensor> const&, KVView const&, KVView const&, unsigned long, unsigned long, unsigned long)",
    "GQA_attention(std::shared_ptr<Tensor> const&, std::shared_ptr<Tensor> const&, std::shared_ptr<Tensor> const&, unsigned long, unsigned long, unsigned long)",
    "apply_rope(std::shared_ptr<Tensor> const&, unsigned long)",
    "reshape_to_heads(std::shared_ptr<Tensor> const&, unsigned long, unsigned long)",
    "quantize_tensor(Tensor const&)",
    "dequantize(QuantizedTensor const&, unsigned long, unsigned long)",
    "matmul_quantized(std::shared_ptr<Tensor> const&, QuantizedTensor const&)",
    "matmul_quantized_range_blocked(float const*, QuantizedTensor const&, float*, unsigned long, unsigned long, unsigned long, unsigned long, unsigned long)",
]


def test_shim_exports_reference_signatures():
    if not os.path.exists(SHIM_LIB):
        subprocess.run(["python", os.path.join(ROOT, "s1-infer_b200", "build.py")], check=True)
    out = subprocess.run(["nm", "-DC", "--defined-only", SHIM_LIB], capture_output=True, text=True).stdout
    missing = [s for s in EXPECTED if s not in out]
    assert not missing, missing


@pytest.mark.gpu
def test_shim_program_on_gpu():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"), "all"], check=True)
    r = subprocess.run([os.path.join(ROOT, "tests", "cpp", "_build", "test_shim")], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout


def test_reference_unit_tests_build_against_shim():
    """`make -C oracle shimtests` compiles the reference's unit tests
    unchanged against the shim wherever the reference sources are present;
    the binaries must then exist (build outputs, never committed)."""
    if not os.path.exists(SHIM_LIB):
        subprocess.run(["python", os.path.join(ROOT, "s1-infer_b200", "build.py")], check=True)
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "shimtests"], capture_output=True,
                       text=True, check=True)
    if "skipping shimtests" in r.stdout:
        pytest.skip("reference sources absent on this machine; the binaries travel prebuilt")
    for name in ("test_kv_block_pool", "test_attention", "test_rope"):
        assert os.path.exists(os.path.join(REF_DIR, f"{name}_on_shim")), name


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["test_kv_block_pool", "test_attention", "test_rope"])
def test_reference_unit_tests_on_shim(name):
    exe = os.path.join(REF_DIR, f"{name}_on_shim")
    assert os.path.exists(exe), ("the reference's tests compiled against the shim are missing: run "
                                 "`make -C oracle shimtests` where the reference sources are present")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "Status: SUCCESS" in r.stdout, r.stdout
