"""The versioned prefix-cache file (format 1).  CPU: a file written by hand
from the documented layout (include/s1kv.h, csrc/prefix_file.cpp) is read
back by s1kv_prefix_file_info, and a flipped byte, a truncated file or a
wrong magic are rejected.  GPU: save from one pool, load into a fresh pool
with its blocks registered in the prefix cache; K/V come back bit for bit
and a prompt with the same tokens shares the loaded blocks."""
import struct

import numpy as np
import pytest


def fnv1a64(b):
    h = 1469598103934665603
    for c in b:
        h = ((h ^ c) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def write_v1(path, layers, hkv, d, n, tokens=None, dtype=0, theta=1e6, rng=None):
    rng = rng or np.random.default_rng(0)
    body = b""
    if tokens is not None:
        body += np.asarray(tokens, np.int32).tobytes()
    kv = rng.standard_normal((layers, 2, n, hkv, d)).astype(np.float32)
    body += kv.tobytes() if dtype == 0 else (kv.view(np.uint32) >> 16).astype(np.uint16).tobytes()
    hdr = struct.pack("<8s8I q f I Q", b"S1KVPFX\0", 1, 64, layers, hkv, d, 16, dtype, 1 if tokens is not None else 0,
                      n, theta, 0, fnv1a64(body))
    assert len(hdr) == 64
    path.write_bytes(hdr + body)
    return kv


def test_file_info_reads_a_hand_written_file(s1kv, tmp_path):
    p = tmp_path / "pre.s1kv"
    write_v1(p, 2, 3, 8, 5, tokens=np.arange(5))
    info = s1kv.prefix_file_info(p)
    assert (info["version"], info["num_layers"], info["num_kv_heads"], info["head_dim"], info["n_tokens"],
            info["has_tokens"], info["dtype"]) == (1, 2, 3, 8, 5, 1, 0)
    assert info["rope_theta"] == 1e6


@pytest.mark.parametrize("damage", ["flip", "truncate", "magic"])
def test_file_info_rejects_damaged_files(s1kv, tmp_path, damage):
    p = tmp_path / "pre.s1kv"
    write_v1(p, 1, 2, 8, 4, tokens=np.arange(4), dtype=1)
    b = bytearray(p.read_bytes())
    if damage == "flip":
        b[100] ^= 0x10
    elif damage == "truncate":
        b = b[:-2]
    else:
        b[0] = ord("X")
    p.write_bytes(bytes(b))
    with pytest.raises(s1kv.S1KVError) as e:
        s1kv.prefix_file_info(p)
    assert e.value.status == s1kv.EINVAL


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_save_load_round_trip_registers_blocks(s1kv, oracle, cuda, tmp_path, dtype):
    import torch
    L, Hkv, D, n = 2, 2, 64, 53
    rng = np.random.default_rng(5)
    tokens = rng.integers(0, 1 << 20, size=n).astype(np.int32)
    src = s1kv.Pool(L, Hkv, D, 64, 16, dtype=dtype)
    with src.batch([7], [n], [0]) as b:
        for layer in range(L):
            b.append(layer, torch.from_numpy(rng.standard_normal((n, Hkv, D)).astype(np.float32)).cuda(),
                     torch.from_numpy(rng.standard_normal((n, Hkv, D)).astype(np.float32)).cuda())
    path = tmp_path / "p.s1kv"
    src.prefix_save_v1(7, path, tokens)
    info = s1kv.prefix_file_info(path)
    assert info["n_tokens"] == n and info["dtype"] == (0 if dtype == "f32" else 1) and info["has_tokens"] == 1
    dst = s1kv.Pool(L, Hkv, D, 64, 16, dtype=dtype, initial_free_list=np.random.default_rng(1).permutation(64))
    assert dst.prefix_load_v1(3, path, register=True) == n
    for layer in range(L):
        for which in (0, 1):
            assert np.array_equal(src.gather(layer, 7, which).cpu().numpy(), dst.gather(layer, 3, which).cpu().numpy())
    # a later prompt with the same tokens shares the loaded full blocks
    hit = dst.prefix_match(4, np.concatenate([tokens, [1, 2, 3]]))
    assert hit == (n // 16) * 16
    assert list(dst.block_table(4)) == list(dst.block_table(3)[: n // 16])
    other = s1kv.Pool(L, Hkv, 128, 64, 16, dtype=dtype)
    with pytest.raises(s1kv.S1KVError):
        other.prefix_load_v1(1, path)
    for pl in (src, dst, other):
        assert pl.check_device() == 0
        pl.close()
