"""The on-disk 12-bit format: save / load round trip, the checks that reject a stale, foreign or
damaged file, and the cache helper that encodes once and reuses the file afterwards."""

import os

import numpy as np

from muse_bf16_proj_b200 import codec12


def _weights(n, k, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w.reshape(-1)[rng.choice(n * k, n * k // 500, replace=False)] = 0.0  # escapes
    return (w.view(np.uint32) >> 16).astype(np.uint16)  # truncation to BF16 bits is fine here


def test_save_load_round_trip(tmp_path):
    wb = _weights(200, 1024, 1)
    enc = codec12.encode(wb)
    key = codec12.weight_key(wb)
    path = os.path.join(tmp_path, "w.m12")
    codec12.save(enc, path, key)
    back = codec12.load(path, key)
    assert back is not None and back.n == enc.n and back.k == enc.k
    for a, b in ((back.planes, enc.planes), (back.bases, enc.bases), (back.esc_ptr, enc.esc_ptr),
                 (back.esc_val, enc.esc_val)):
        assert np.array_equal(a, b)
    assert np.array_equal(codec12.decode(back), wb)
    assert os.path.getsize(path) % 256 == 0


def test_load_rejects_foreign_stale_and_damaged_files(tmp_path):
    wb = _weights(128, 512, 2)
    enc = codec12.encode(wb)
    key = codec12.weight_key(wb)
    path = os.path.join(tmp_path, "w.m12")
    codec12.save(enc, path, key)
    assert codec12.load(path, "0" * 64) is None                     # another weight's key
    assert codec12.load(os.path.join(tmp_path, "missing.m12")) is None
    raw = bytearray(open(path, "rb").read())
    damaged = os.path.join(tmp_path, "d.m12")
    open(damaged, "wb").write(raw[: len(raw) // 2])                  # truncated
    assert codec12.load(damaged, key) is None
    v2 = bytes(raw).replace(b'"version": 1', b'"version": 9')      # another format version
    open(damaged, "wb").write(v2)
    assert codec12.load(damaged, key) is None
    assert codec12.weight_key(wb) != codec12.weight_key(wb.reshape(256, 256))  # the shape is in the key


def test_encode_cached_reuses_the_file(tmp_path):
    wb = _weights(256, 1024, 3)
    enc1, cached1 = codec12.encode_cached(wb, str(tmp_path))
    enc2, cached2 = codec12.encode_cached(wb, str(tmp_path))
    assert not cached1 and cached2
    assert np.array_equal(enc1.planes, enc2.planes) and np.array_equal(enc1.esc_val, enc2.esc_val)
    files = os.listdir(tmp_path)
    assert files == [f"{codec12.weight_key(wb)}.m12"]
    other = wb.copy()
    other[0, 0] ^= 1
    _, cached3 = codec12.encode_cached(other, str(tmp_path))
    assert not cached3 and len(os.listdir(tmp_path)) == 2
