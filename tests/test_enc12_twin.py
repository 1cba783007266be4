"""The device 12-bit encoder's program, replayed on the host (tests/enc12_twin.cpp: the kernels'
grids, per-lane steps and index arithmetic over the shared rules in csrc/enc12_core.h), against the
host encoder muse_encode12 bit for bit: planes, window bases, escape offsets and entries. Ragged N,
every BF16 bit pattern, escape-dense tiles and a short escape buffer (writes past it skipped, none
out of bounds). The kernels themselves run against the same encoder in test_zy_gpu_encode12.py."""

import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

from muse_bf16_proj_b200 import codec12

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def twin(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    out = str(tmp_path_factory.mktemp("enc12") / "libenc12_twin.so")
    subprocess.run([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-o", out, os.path.join(HERE, "enc12_twin.cpp")],
                   check=True, capture_output=True)
    lib = ctypes.CDLL(out)
    lib.enc12_twin.restype = ctypes.c_int64
    lib.enc12_twin.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64] + [ctypes.c_void_p] * 4 + [ctypes.c_int64]
    return lib


def _run(twin, w: np.ndarray, esc_cap: int | None = None, guard: int = 64):
    n, k = w.shape
    planes = np.full(n * k * 3 // 2, 0xEE, np.uint8)
    bases = np.full(-(-n // 128) * (k // 128), 0xEE, np.uint8)
    esc_ptr = np.full(n + 1, -7, np.int32)
    cap = n * k if esc_cap is None else esc_cap
    esc_val = np.full(cap + guard, 0xDEADBEEF, np.uint32)  # the guard words must stay untouched
    p = lambda a: a.ctypes.data  # noqa: E731
    skipped = twin.enc12_twin(p(w), n, k, p(planes), p(bases), p(esc_ptr), p(esc_val), cap)
    assert (esc_val[cap:] == 0xDEADBEEF).all(), "an escape was written past the buffer"
    return planes, bases, esc_ptr, esc_val[:cap], skipped


def _same_as_host(twin, w: np.ndarray):
    enc = codec12.encode(w)
    planes, bases, esc_ptr, esc_val, skipped = _run(twin, w)
    assert skipped == 0
    assert np.array_equal(bases, enc.bases.reshape(-1)), "window bases"
    assert np.array_equal(esc_ptr, enc.esc_ptr), "escape offsets"
    assert np.array_equal(esc_val[: enc.n_esc], enc.esc_val), "escape entries"
    assert np.array_equal(planes, enc.planes), "planes"
    return enc


def _normal(n, k, seed, inject=0.0):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if inject:
        idx = rng.choice(n * k, int(n * k * inject), replace=False)
        flat = w.reshape(-1)
        flat[idx[: len(idx) // 2]] = 0.0
        flat[idx[len(idx) // 2:]] *= 50.0
    bits = w.view(np.uint32)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even


@pytest.mark.parametrize("n,k,inject", [(1, 512, 0.0), (300, 1024, 0.001), (128, 2048, 0.01), (257, 512, 0.05)])
def test_twin_matches_host_encoder(twin, n, k, inject):
    enc = _same_as_host(twin, _normal(n, k, n * 7 + k, inject))
    if inject >= 0.01:
        assert enc.n_esc > 0


def test_twin_every_bf16_pattern(twin):
    w = np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(128, 512)
    enc = _same_as_host(twin, w)
    assert enc.n_esc > 0


def test_twin_escape_dense_rows(twin):
    rng = np.random.default_rng(3)
    w = _normal(200, 1024, 5)
    w[17] = rng.integers(0, 65536, 1024, dtype=np.uint16)  # a row of random bits: mostly escapes
    w[130, ::3] = 0x7F80  # +inf every third weight of a row in the second tile
    _same_as_host(twin, w)


def test_twin_short_escape_buffer_skips_and_counts(twin):
    w = _normal(64, 512, 9, inject=0.05)
    enc = codec12.encode(w)
    cap = enc.n_esc // 2
    _, _, esc_ptr, esc_val, skipped = _run(twin, w, esc_cap=cap)
    assert skipped == enc.n_esc - cap
    assert np.array_equal(esc_val, enc.esc_val[:cap])
    assert np.array_equal(esc_ptr, enc.esc_ptr)


def test_twin_every_window_base(twin):
    """The device program under each of the 121 window bases (0..120), every tile forced to it by
    filler weights, all 65,536 BF16 patterns in each matrix."""
    from test_codec12 import _forced_base

    perm = np.random.default_rng(1).permutation(65536)
    for c in range(121):
        enc = _same_as_host(twin, _forced_base(c, perm))
        assert (enc.bases == c).all()
