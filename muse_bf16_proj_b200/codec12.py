"""Host-side 12-bit lossless weight codec (the C ABI's muse_encode12 / muse_decode12).

``encode(w)`` replaces the reference's ``nf12_pack_cuda`` (submission.py:591-626): it packs a
BF16 [N, K] matrix into 12 bits a weight with a window base per 128 x 128 tile, checks the round
trip bit for bit (the reference asserts the same, submission.py:611-617) and returns numpy arrays
ready to copy to the device.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib

UNIT = 512
UNIT_BYTES = 768
TILE = 128
MAX_ESCAPE_FRACTION = 0.01  # as the reference's NF12_MAX_ESCAPE_FRACTION (submission.py:127)


@dataclass
class Encoded12:
    planes: np.ndarray   # u8 [N * K * 3 / 2]
    bases: np.ndarray    # u8 [ceil(N/128), K/128]
    esc_ptr: np.ndarray  # i32 [N + 1]
    esc_val: np.ndarray  # u32 [n_esc]
    n: int
    k: int

    @property
    def n_esc(self) -> int:
        return int(self.esc_val.size)

    @property
    def escape_fraction(self) -> float:
        return self.n_esc / float(self.n * self.k)

    @property
    def nbytes(self) -> int:
        return self.planes.nbytes + self.bases.nbytes + self.esc_ptr.nbytes + self.esc_val.nbytes


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def encode(w_bits: np.ndarray, threads: int = 0, verify: bool = True) -> Encoded12:
    """BF16 bits (uint16 [N, K], C-contiguous) -> Encoded12. ``verify`` decodes and compares."""
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    n, k = w_bits.shape
    lib = _lib.load()
    pb, bb = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(lib.muse_encode12_sizes(n, k, ctypes.byref(pb), ctypes.byref(bb)))
    planes = np.empty(pb.value, dtype=np.uint8)
    bases = np.empty(bb.value, dtype=np.uint8)
    esc_ptr = np.empty(n + 1, dtype=np.int32)
    cap = max(1024, (n * k) // 256)
    esc_val = np.empty(cap, dtype=np.uint32)
    n_esc = ctypes.c_int64()
    rc = lib.muse_encode12(_ptr(w_bits), n, k, _ptr(planes), _ptr(bases), _ptr(esc_ptr), _ptr(esc_val), cap,
                           ctypes.byref(n_esc), threads)
    if rc == -4 and n_esc.value > cap:
        cap = int(n_esc.value)
        esc_val = np.empty(cap, dtype=np.uint32)
        rc = lib.muse_encode12(_ptr(w_bits), n, k, _ptr(planes), _ptr(bases), _ptr(esc_ptr), _ptr(esc_val), cap,
                               ctypes.byref(n_esc), threads)
    _lib.check(rc)
    enc = Encoded12(planes, bases.reshape(-(-n // TILE), k // TILE), esc_ptr, esc_val[: n_esc.value].copy(), n, k)
    if verify:
        back = decode(enc, threads)
        if not np.array_equal(back, w_bits):
            bad = int(np.count_nonzero(back != w_bits))
            raise AssertionError(f"12-bit codec round trip mismatch in {bad} weights")
    return enc


def decode(enc: Encoded12, threads: int = 0) -> np.ndarray:
    out = np.empty((enc.n, enc.k), dtype=np.uint16)
    esc = enc.esc_val if enc.esc_val.size else np.zeros(1, dtype=np.uint32)
    _lib.check(_lib.load().muse_decode12(_ptr(enc.planes), _ptr(enc.bases), _ptr(enc.esc_ptr), _ptr(esc),
                                         enc.n, enc.k, _ptr(out), threads))
    return out


def plane_bytes(n: int, k: int) -> int:
    """HBM bytes the 12-bit GEMV streams for the planes alone."""
    return n * k * 3 // 2
