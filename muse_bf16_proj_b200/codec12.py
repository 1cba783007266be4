"""Host-side 12-bit lossless weight codec (the C ABI's muse_encode12 / muse_decode12) and its
on-disk format (``save`` / ``load`` / ``encode_cached``: encode once, reuse across processes).

``encode(w)`` replaces the reference's ``nf12_pack_cuda`` (submission.py:591-626): it packs a
BF16 [N, K] matrix into 12 bits a weight with a window base per 128 x 128 tile, checks the round
trip bit for bit (the reference asserts the same, submission.py:611-617) and returns numpy arrays
ready to copy to the device.
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import os
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


# ---- on-disk format --------------------------------------------------------------------------
#
# One file per encoded weight, `<sha256 of the BF16 weight bits>.m12`: a 1024-byte header (JSON,
# NUL padded: magic, format version, n, k, escape count, the weight's sha256 and each array's
# offset and length), then the planes, bases, esc_ptr and esc_val arrays, each starting on a
# 256-byte boundary, little-endian as in memory. Loading checks the magic, the version, the sizes
# and the weight hash; a file that fails any check is ignored (the caller re-encodes).

FILE_MAGIC = "muse-12bit"
FILE_VERSION = 1
_HEADER = 1024
_ALIGN = 256


def weight_key(w_bits: np.ndarray) -> str:
    """The cache key of a BF16 weight: sha256 of its bits and shape."""
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    h = hashlib.sha256(np.asarray(w_bits.shape, dtype=np.int64).tobytes())
    h.update(w_bits.tobytes())
    return h.hexdigest()


def save(enc: Encoded12, path: str, key: str) -> None:
    """Writes `enc` (the encoding of the weight whose weight_key is `key`) to `path` atomically."""
    arrays = [("planes", enc.planes), ("bases", np.ascontiguousarray(enc.bases).reshape(-1)),
              ("esc_ptr", enc.esc_ptr), ("esc_val", enc.esc_val)]
    layout, off = {}, _HEADER
    for name, a in arrays:
        layout[name] = [off, int(a.nbytes)]
        off += -(-int(a.nbytes) // _ALIGN) * _ALIGN
    header = json.dumps({"magic": FILE_MAGIC, "version": FILE_VERSION, "n": enc.n, "k": enc.k,
                         "n_esc": enc.n_esc, "key": key, "arrays": layout}).encode()
    if len(header) >= _HEADER:
        raise ValueError("12-bit file header does not fit")
    tmp = f"{path}.tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(header.ljust(_HEADER, b"\0"))
        for name, a in arrays:
            f.seek(layout[name][0])
            f.write(np.ascontiguousarray(a).tobytes())
        f.truncate(off)
    os.replace(tmp, path)


def load(path: str, key: str | None = None) -> Encoded12 | None:
    """The encoding stored at `path`, or None when the file is missing, of another format version,
    inconsistent, or (with `key`) of another weight."""
    try:
        with open(path, "rb") as f:
            raw = f.read()
    except OSError:
        return None
    try:
        hdr = json.loads(raw[:_HEADER].rstrip(b"\0").decode())
        if hdr.get("magic") != FILE_MAGIC or hdr.get("version") != FILE_VERSION:
            return None
        if key is not None and hdr.get("key") != key:
            return None
        n, k, n_esc = int(hdr["n"]), int(hdr["k"]), int(hdr["n_esc"])

        def arr(name, dtype, count):
            off, nbytes = hdr["arrays"][name]
            if nbytes != count * np.dtype(dtype).itemsize or off + nbytes > len(raw):
                raise ValueError(name)
            return np.frombuffer(raw, dtype=dtype, count=count, offset=off).copy()

        planes = arr("planes", np.uint8, n * k * 3 // 2)
        bases = arr("bases", np.uint8, -(-n // TILE) * (k // TILE)).reshape(-(-n // TILE), k // TILE)
        esc_ptr = arr("esc_ptr", np.int32, n + 1)
        esc_val = arr("esc_val", np.uint32, n_esc)
        if esc_ptr[0] != 0 or esc_ptr[-1] != n_esc or np.any(np.diff(esc_ptr) < 0):
            return None
        return Encoded12(planes, bases, esc_ptr, esc_val, n, k)
    except (ValueError, KeyError, TypeError, json.JSONDecodeError, UnicodeDecodeError):
        return None


def encode_cached(w_bits: np.ndarray, cache_dir: str | None, threads: int = 0) -> tuple[Encoded12, bool]:
    """(encoding, from_cache): the encoding of `w_bits` from `cache_dir` when a valid file for this
    exact weight is there, else a fresh (round-trip checked) encoding, saved there when given."""
    if not cache_dir:
        return encode(w_bits, threads), False
    key = weight_key(w_bits)
    path = os.path.join(cache_dir, f"{key}.m12")
    enc = load(path, key)
    if enc is not None and enc.n == w_bits.shape[0] and enc.k == w_bits.shape[1]:
        return enc, True
    enc = encode(w_bits, threads)
    os.makedirs(cache_dir, exist_ok=True)
    save(enc, path, key)
    return enc, False


def plane_bytes(n: int, k: int) -> int:
    """HBM bytes the 12-bit GEMV streams for the planes alone."""
    return n * k * 3 // 2
