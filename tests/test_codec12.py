"""The product's host 12-bit encoder (C ABI) against the numpy oracle, and its round trip."""

import numpy as np
import pytest
import torch

from muse_bf16_proj_b200 import _lib, codec12
from muse_bf16_proj_b200 import contract as C
from oracle import codec12_ref as Q


def assert_same(enc, ref):
    assert np.array_equal(enc.planes, ref["planes"])
    assert np.array_equal(enc.bases, ref["bases"])
    assert np.array_equal(enc.esc_ptr, ref["esc_ptr"])
    assert np.array_equal(enc.esc_val, ref["esc_val"])


@pytest.mark.parametrize("n,k", [(1, 512), (16, 1024), (130, 1536), (257, 2048), (128, 65536 // 8)])
def test_encoder_matches_oracle_random(n, k):
    rng = np.random.default_rng(n * 7 + k)
    w = (rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    wb = (w.view(np.uint32) >> 16).astype(np.uint16)
    assert_same(codec12.encode(wb), Q.encode_tiles(wb))


def test_all_bf16_bit_patterns_round_trip():
    """Every one of the 65,536 BF16 patterns (NaNs, infinities, subnormals, +-0) survives."""
    wb = np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(128, 512)
    enc = codec12.encode(wb)  # verify=True decodes and compares bit for bit
    assert_same(enc, Q.encode_tiles(wb))
    assert np.array_equal(Q.decode_tiles(enc.planes, enc.bases, enc.esc_ptr, enc.esc_val, 128, 512), wb)
    # shuffled across tiles, so windows differ per tile
    perm = np.random.default_rng(0).permutation(65536)
    wb2 = wb.reshape(-1)[perm].reshape(256, 256 * 1).repeat(2, axis=1)
    enc2 = codec12.encode(wb2)
    assert_same(enc2, Q.encode_tiles(wb2))


def _forced_base(c: int, perm: np.ndarray) -> np.ndarray:
    """W [128, 1024]: the even columns hold all 65,536 BF16 patterns (shuffled by `perm`), the odd
    columns filler weights whose E7 spreads evenly over [c, c + 7]. Per 128 x 128 tile the filler
    (8,192 weights) outweighs the patterns (about 64 per E7 value), so every tile's base is c."""
    rng = np.random.default_rng(c)
    w = np.empty((128, 1024), np.uint16)
    w[:, 0::2] = np.arange(65536, dtype=np.uint32)[perm].astype(np.uint16).reshape(128, 512)
    e7 = c + (np.arange(128 * 512) % 8)
    filler = (rng.integers(0, 2, 128 * 512) << 15) | (e7 << 8) | rng.integers(0, 256, 128 * 512)
    w[:, 1::2] = filler.astype(np.uint16).reshape(128, 512)
    return w


def test_all_bf16_patterns_under_every_window_base():
    """All 65,536 patterns round-trip bit for bit under each of the 121 window bases a tile can
    take (0..120), the encoder choosing the forced base in every tile; three bases also against
    the oracle's encoder and decoder."""
    perm = np.random.default_rng(1).permutation(65536)
    for c in range(121):
        wb = _forced_base(c, perm)
        enc = codec12.encode(wb)  # verify=True decodes and compares bit for bit
        assert (enc.bases == c).all(), f"base {c}: got {np.unique(enc.bases)}"
        if c in (0, 60, 120):
            assert_same(enc, Q.encode_tiles(wb))
            assert np.array_equal(Q.decode_tiles(enc.planes, enc.bases, enc.esc_ptr, enc.esc_val, 128, 1024), wb)


def test_baseline_injected_weights_escape_fraction():
    w = C.generate_baseline_weight("qkv_decode", 11, device="cpu", recipe="inject")
    wb = w.view(torch.int16).numpy().view(np.uint16)
    enc = codec12.encode(wb)
    assert_same(enc, Q.encode_tiles(wb))
    # ~0.1 % injected zeros/outliers are escapes; per-tile windows leave almost no natural ones
    assert 0.0008 < enc.escape_fraction < 0.0015
    assert enc.planes.nbytes * 8 / wb.size == 12.0


def test_ragged_rows_and_tile_edges():
    rng = np.random.default_rng(5)
    n, k = 200, 1024
    w = rng.standard_normal((n, k)).astype(np.float32)
    w[:100] *= 1e-3   # rows in the same tile with very different scales
    w[150:, 512:] *= 1e4
    wb = (w.view(np.uint32) >> 16).astype(np.uint16)
    enc = codec12.encode(wb)
    assert_same(enc, Q.encode_tiles(wb))
    assert enc.bases.shape == (2, 8)


def test_encoder_rejects_bad_shapes_and_capacity():
    lib = _lib.load()
    import ctypes
    pb, bb = ctypes.c_int64(), ctypes.c_int64()
    assert lib.muse_encode12_sizes(4, 1000, ctypes.byref(pb), ctypes.byref(bb)) == -3
    assert lib.muse_encode12_sizes(4, 500, ctypes.byref(pb), ctypes.byref(bb)) == -1
    assert lib.muse_encode12_sizes(0, 512, ctypes.byref(pb), ctypes.byref(bb)) == -1
    assert lib.muse_encode12_sizes(4, 512 * 200, ctypes.byref(pb), ctypes.byref(bb)) == -3
    assert lib.muse_encode12_sizes(3, 1024, ctypes.byref(pb), ctypes.byref(bb)) == 0
    assert pb.value == 3 * 1024 * 3 // 2 and bb.value == 8
    # capacity: all-zero weights are all escapes except the window... force escapes with a mix
    wb = np.zeros((2, 512), dtype=np.uint16)
    wb[:, ::2] = 0x3F80  # 1.0; zeros fall outside the window
    planes = np.empty(2 * 512 * 3 // 2, np.uint8)
    bases = np.empty(4, np.uint8)
    esc_ptr = np.empty(3, np.int32)
    esc_val = np.empty(4, np.uint32)
    n_esc = ctypes.c_int64()
    rc = lib.muse_encode12(wb.ctypes.data, 2, 512, planes.ctypes.data, bases.ctypes.data, esc_ptr.ctypes.data,
                           esc_val.ctypes.data, 4, ctypes.byref(n_esc), 1)
    assert rc == -4 and n_esc.value == 512
    assert b"capacity" in lib.muse_last_error()
    assert lib.muse_encode12(None, 2, 512, planes.ctypes.data, bases.ctypes.data, esc_ptr.ctypes.data,
                             esc_val.ctypes.data, 4, ctypes.byref(n_esc), 1) == -1


def test_escapes_are_stored_as_the_placeholder():
    """An escaped weight's plane bytes are low byte 0 and code 0, so every decoder (the tensor-core
    path's in-place decode and the register-decoding GEMV's correction) reads it as the tile's
    placeholder BF16 base << 8 until its true bits are applied."""
    w = C.generate_baseline_weight("qkv_decode", 12, device="cpu", recipe="inject")
    wb = w.view(torch.int16).numpy().view(np.uint16)
    n, k = wb.shape
    enc = codec12.encode(wb)
    units = enc.planes.reshape(n, k // 512, 768)
    low = units[:, :, :512].reshape(n, k)
    cb = units[:, :, 512:].reshape(n, k // 2)
    code = np.empty((n, k), dtype=np.uint8)
    code[:, 0::2] = cb & 15
    code[:, 1::2] = cb >> 4
    rows = np.repeat(np.arange(n), np.diff(enc.esc_ptr))
    ks = (enc.esc_val >> 16).astype(np.int64)
    assert rows.size > 0
    assert not low[rows, ks].any() and not code[rows, ks].any()
