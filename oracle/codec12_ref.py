"""numpy restatement of the 12-bit lossless BF16 weight codecs. TEST INFRASTRUCTURE ONLY.

A BF16 weight is  s | e7..e1 | e0 m6..m0.  E7 = its high byte without the sign (7 bits). A window
base c0 covers E7 in [c0, c0 + 7] (16 full exponents, because e0 rides in the low byte). A weight
inside the window is kept as its low byte (8 bits, verbatim) plus a 4-bit code s << 3 | (E7 - c0);
it rebuilds as  high = (code & 8) << 4 | (c0 + (code & 7)),  bits = high << 8 | low.  A weight
outside the window is stored as low = 0, code = 0 (it rebuilds to the placeholder bf16(c0 << 8))
and listed as an escape.

Two formats, both lossless:

``pack_reference``: the reference's ``nf12_pack_cuda`` (submission.py:591-626): ONE c0 per matrix,
the 8-wide E7 window holding the most weights (first such window on ties, like torch.argmax); planes
lo [N, K] and nib [N, K/2] (low nibble = even k); per-row CSR escapes (esc_ptr, esc_k, esc_delta =
true value - placeholder, FP32). Rejects K % 512, N % 16 and more than 1 % escapes, as the
reference does (submission.py:127, 596-606).

``encode_tiles``: the B200 build's format. c0 is chosen per 128 x 128 tile by the same rule. The
HBM layout streams one row at a time in 768-byte units of 512 weights: 512 low bytes, then 256 code
bytes (byte j = code[2j] | code[2j+1] << 4). Bases u8 [ceil(N/128)][K/128]. Escapes as a per-row
CSR of u32 entries k << 16 | true BF16 bits (k ascending within a row; K <= 65536).
"""

from __future__ import annotations

import numpy as np

UNIT = 512          # weights per streamed unit
UNIT_BYTES = 768    # 512 low bytes + 256 code bytes
TILE_R = 128
TILE_K = 128
MAX_ESCAPE_FRACTION = 0.01  # submission.py:127


def e7_of(bits: np.ndarray) -> np.ndarray:
    return ((np.asarray(bits, dtype=np.uint16) >> 8) & 0x7F).astype(np.int32)


def best_window(counts: np.ndarray) -> np.ndarray:
    """counts [..., 128] of E7 -> c0 [...]: the first c in 0..120 maximising counts[c:c+8].sum()."""
    csum = np.concatenate([np.zeros(counts.shape[:-1] + (1,), np.int64), np.cumsum(counts, -1, dtype=np.int64)], -1)
    windows = csum[..., 8:] - csum[..., :-8]          # [..., 121]
    return np.argmax(windows, axis=-1).astype(np.int32)


def decode_window(code: np.ndarray, low: np.ndarray, c0) -> np.ndarray:
    """code (0..15), low byte, window base -> BF16 bits."""
    code = np.asarray(code, dtype=np.int32)
    hb = ((code & 8) << 4) | (np.asarray(c0, dtype=np.int32) + (code & 7))
    return ((hb << 8) | np.asarray(low, dtype=np.int32)).astype(np.uint16)


# ---------------------------------------------------------------------------------------------
# The reference's per-matrix format (submission.py:591-626).
# ---------------------------------------------------------------------------------------------

def pack_reference(w_bits: np.ndarray):
    """BF16 bits [N, K] -> dict(lo, nib, c0, esc_ptr, esc_k, esc_delta, escapes), or None when the
    reference would refuse (K % 512, N % 16, or more than 1 % escapes)."""
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    n, k = w_bits.shape
    if k % 512 or n % 16:
        return None
    e7 = e7_of(w_bits)
    counts = np.bincount(e7.ravel(), minlength=128).astype(np.int64)
    c0 = int(best_window(counts))
    inside = (e7 >= c0) & (e7 < c0 + 8)
    n_esc = int((~inside).sum())
    if n_esc > MAX_ESCAPE_FRACTION * w_bits.size:
        return None
    bits = w_bits.astype(np.int32)
    code = np.where(inside, ((bits >> 15) << 3) | (e7 - c0), 0)
    lo = np.where(inside, bits & 0xFF, 0).astype(np.uint8)
    nib = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    placeholder = np.array([c0 << 24], dtype=np.uint32).view(np.float32)[0]
    rows, ks = np.nonzero(~inside)
    esc_ptr = np.zeros(n + 1, dtype=np.int32)
    esc_ptr[1:] = np.cumsum(np.bincount(rows, minlength=n)).astype(np.int32)
    true_vals = (w_bits[rows, ks].astype(np.uint32) << 16).view(np.float32)
    esc_delta = (true_vals - placeholder).astype(np.float32)
    return {"lo": lo, "nib": nib, "c0": c0, "esc_ptr": esc_ptr, "esc_k": ks.astype(np.int32),
            "esc_delta": esc_delta, "escapes": n_esc}


def unpack_reference(p: dict) -> np.ndarray:
    """Rebuild BF16 bits from ``pack_reference``'s planes and escapes (exact)."""
    lo, nib, c0 = p["lo"], p["nib"], p["c0"]
    n, k = lo.shape
    code = np.empty((n, k), dtype=np.int32)
    code[:, 0::2] = nib & 0xF
    code[:, 1::2] = nib >> 4
    bits = decode_window(code, lo, c0)
    placeholder = np.array([c0 << 24], dtype=np.uint32).view(np.float32)[0]
    for r in range(n):
        for e in range(p["esc_ptr"][r], p["esc_ptr"][r + 1]):
            val = np.float32(placeholder + p["esc_delta"][e])
            bits[r, p["esc_k"][e]] = np.array([val], dtype=np.float32).view(np.uint32)[0] >> 16
    return bits


# ---------------------------------------------------------------------------------------------
# The build's per-tile format.
# ---------------------------------------------------------------------------------------------

def tile_bases(w_bits: np.ndarray, tile_r: int = TILE_R, tile_k: int = TILE_K) -> np.ndarray:
    """c0 per tile: u8 [ceil(N / tile_r)][ceil(K / tile_k)] (ragged edge tiles count what they hold)."""
    n, k = w_bits.shape
    tr, tk = -(-n // tile_r), -(-k // tile_k)
    e7 = e7_of(w_bits)
    tile_id = (np.arange(n)[:, None] // tile_r) * tk + (np.arange(k)[None, :] // tile_k)
    counts = np.bincount((tile_id * 128 + e7).ravel(), minlength=tr * tk * 128).reshape(tr, tk, 128)
    return best_window(counts).astype(np.uint8)


def encode_tiles(w_bits: np.ndarray, tile_r: int = TILE_R, tile_k: int = TILE_K) -> dict:
    """BF16 bits [N, K] -> dict(planes u8 [N * K * 3 / 2], bases, esc_ptr, esc_val, lo, code, inside)."""
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    n, k = w_bits.shape
    if k % UNIT or k > 65536 or n < 1:
        raise ValueError("encode_tiles needs K % 512 == 0, K <= 65536, N >= 1")
    bases = tile_bases(w_bits, tile_r, tile_k)
    c0 = bases[(np.arange(n) // tile_r)[:, None], (np.arange(k) // tile_k)[None, :]].astype(np.int32)
    e7 = e7_of(w_bits)
    inside = (e7 >= c0) & (e7 < c0 + 8)
    bits = w_bits.astype(np.int32)
    code = np.where(inside, ((bits >> 15) << 3) | (e7 - c0), 0).astype(np.uint8)
    lo = np.where(inside, bits & 0xFF, 0).astype(np.uint8)
    units = k // UNIT
    planes = np.empty((n, units, UNIT_BYTES), dtype=np.uint8)
    planes[:, :, :UNIT] = lo.reshape(n, units, UNIT)
    c = code.reshape(n, units, UNIT)
    planes[:, :, UNIT:] = c[:, :, 0::2] | (c[:, :, 1::2] << 4)
    rows, ks = np.nonzero(~inside)
    esc_ptr = np.zeros(n + 1, dtype=np.int32)
    esc_ptr[1:] = np.cumsum(np.bincount(rows, minlength=n)).astype(np.int32)
    esc_val = ((ks.astype(np.uint32) << 16) | w_bits[rows, ks].astype(np.uint32)).astype(np.uint32)
    return {"planes": planes.reshape(-1), "bases": bases, "esc_ptr": esc_ptr, "esc_val": esc_val,
            "lo": lo, "code": code, "inside": inside, "n": n, "k": k}


def decode_tiles(planes: np.ndarray, bases: np.ndarray, esc_ptr: np.ndarray, esc_val: np.ndarray,
                 n: int, k: int, tile_r: int = TILE_R, tile_k: int = TILE_K) -> np.ndarray:
    """Rebuild BF16 bits [N, K] from the per-tile format (exact, escapes included)."""
    units = k // UNIT
    p = np.asarray(planes, dtype=np.uint8).reshape(n, units, UNIT_BYTES)
    lo = p[:, :, :UNIT].reshape(n, k)
    nib = p[:, :, UNIT:].reshape(n, k // 2)
    code = np.empty((n, k), dtype=np.int32)
    code[:, 0::2] = nib & 0xF
    code[:, 1::2] = nib >> 4
    c0 = bases[(np.arange(n) // tile_r)[:, None], (np.arange(k) // tile_k)[None, :]].astype(np.int32)
    bits = decode_window(code, lo, c0)
    rows = np.repeat(np.arange(n), np.diff(esc_ptr))
    ks = (np.asarray(esc_val, dtype=np.uint32) >> 16).astype(np.int64)
    bits[rows, ks] = (np.asarray(esc_val, dtype=np.uint32) & 0xFFFF).astype(np.uint16)
    return bits


def placeholder_bits(c0) -> np.ndarray:
    """The BF16 bits an escaped weight decodes to before its correction: c0 << 8."""
    return (np.asarray(c0, dtype=np.uint32) << 8).astype(np.uint16)


def gemv_12b(planes, bases, esc_ptr, esc_val, n, k, x_bits) -> np.ndarray:
    """FP64 x @ decode(W).T through the 12-bit format (equal to the plain product on exact decode)."""
    from .contract_ref import bf16_to_f32
    w = decode_tiles(planes, bases, esc_ptr, esc_val, n, k)
    return bf16_to_f32(x_bits).astype(np.float64) @ bf16_to_f32(w).astype(np.float64).T
