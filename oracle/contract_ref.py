"""numpy restatement of the reference's FP64 product and output checks. TEST INFRASTRUCTURE ONLY.

- ``ref_kernel``: reference.py:72-76 — out = x.double() @ W[:n].double().T, then to BF16. torch
  converts FP64 to BF16 through FP32 (two round-to-nearest-even steps); this restatement does the
  same, so the BF16 bits match the reference's (pinned by the golden hashes).
- ``compare``: checks.py:31-55 — relative L2 over the whole output <= tol, every row <= 5 x tol
  against max(row norm, 0.1 x mean row norm), no NaN/Inf, same shape.
- ``check_implementation``: reference.py:84-99 — the above plus probe rows (a single nonzero,
  power-of-two input entry, so the output row is a scaled weight column) within 1e-3.

Arrays are numpy: BF16 tensors are carried as their raw ``uint16`` bits.
"""

from __future__ import annotations

import numpy as np

REL_L2_TOL = 1e-2   # reference.py:27
ROUTER_TOL = 1e-4   # reference.py:29
PROBE_TOL = 1e-3    # reference.py:34
ROW_FACTOR = 5.0    # checks.py:14
ROW_NORM_FLOOR = 0.1  # checks.py:17


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """BF16 bits (uint16) -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(values: np.ndarray) -> np.ndarray:
    """float32 -> BF16 bits, round to nearest even; NaN -> 0x7FC0."""
    f = np.ascontiguousarray(values, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(f), np.uint16(0x7FC0), rounded)


def f64_to_bf16(values: np.ndarray) -> np.ndarray:
    """float64 -> BF16 bits the way torch does it: to float32 first, then to BF16."""
    return f32_to_bf16(np.asarray(values, dtype=np.float64).astype(np.float32))


def ref_product(x_bits: np.ndarray, w_bits: np.ndarray, n: int | None = None) -> np.ndarray:
    """FP64 x @ W[:n].T (float64 array, before rounding)."""
    x = bf16_to_f32(x_bits).astype(np.float64)
    w = bf16_to_f32(w_bits if n is None else w_bits[:n]).astype(np.float64)
    return x @ w.T


def ref_kernel(x_bits: np.ndarray, w_bits: np.ndarray, n: int | None = None) -> np.ndarray:
    """reference.py:72-76 for the BF16 layers: BF16 bits of x @ W[:n].T computed in FP64."""
    return f64_to_bf16(ref_product(x_bits, w_bits, n))


def relative_l2(a: np.ndarray, b: np.ndarray) -> float:
    """|a - b| / |b| (checks.py:20-22), on float values."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-12))


def compare(out_f: np.ndarray, ref_f: np.ndarray, tol: float) -> tuple[bool, str, dict]:
    """checks.py:31-55 on float values; also returns the error figures it computed."""
    out = np.asarray(out_f, dtype=np.float64)
    ref = np.asarray(ref_f, dtype=np.float64)
    stats = {"rel_l2": None, "worst_row": None, "max_abs": None}
    if out.shape != ref.shape:
        return False, f"expected {ref.shape}, got {out.shape}", stats
    if not np.isfinite(out).all():
        return False, "output contains NaN or Inf", stats
    diff = out - ref
    err = float(np.linalg.norm(diff) / max(np.linalg.norm(ref), 1e-12))
    stats["rel_l2"] = err
    stats["max_abs"] = float(np.abs(diff).max()) if diff.size else 0.0
    if err > tol:
        return False, f"relative L2 error {err:.3e} > {tol:g}", stats
    rows_diff = np.linalg.norm(diff.reshape(-1, ref.shape[-1]), axis=-1)
    rows_ref = np.linalg.norm(ref.reshape(-1, ref.shape[-1]), axis=-1)
    floor = max(ROW_NORM_FLOOR * float(rows_ref.mean()), 1e-12)
    row_err = rows_diff / np.maximum(rows_ref, floor)
    worst = int(row_err.argmax())
    stats["worst_row"] = float(row_err[worst])
    if row_err[worst] > ROW_FACTOR * tol:
        return False, (f"relative L2 error {err:.3e}, but row {worst} is off by {row_err[worst]:.3e}"
                       f" > {ROW_FACTOR:g} x {tol:g}"), stats
    return True, f"relative L2 error {err:.3e} (worst row {row_err[worst]:.3e})", stats


def probe_rows(x_bits: np.ndarray) -> np.ndarray:
    """reference.py:79-81: rows of x with exactly one nonzero entry (+0 and -0 both count as 0)."""
    nonzero = (np.asarray(x_bits, dtype=np.uint16) & 0x7FFF) != 0
    return np.nonzero(nonzero.sum(-1) == 1)[0]


def check_implementation(x_bits: np.ndarray, w_bits: np.ndarray, out_bits: np.ndarray, n: int | None = None,
                         tol: float = REL_L2_TOL, ref_bits: np.ndarray | None = None) -> tuple[bool, str, dict]:
    """reference.py:84-99 for a BF16 layer: ``out_bits`` (BF16 bits [M, n]) against the FP64
    reference, then every probe row within PROBE_TOL."""
    if ref_bits is None:
        ref_bits = ref_kernel(x_bits, w_bits, n)
    ref = bf16_to_f32(ref_bits)
    out = bf16_to_f32(out_bits)
    ok, msg, stats = compare(out, ref, tol)
    rows = probe_rows(x_bits)
    stats["probe_rows"] = int(len(rows))
    if not ok or not len(rows):
        return ok, msg, stats
    d = np.linalg.norm(out[rows].astype(np.float64) - ref[rows].astype(np.float64), axis=-1)
    r = np.maximum(np.linalg.norm(ref[rows].astype(np.float64), axis=-1), 1e-30)
    diff = d / r
    worst = int(diff.argmax())
    stats["probe_worst"] = float(diff[worst])
    if diff[worst] > PROBE_TOL:
        return False, (f"{msg}, but probe row {int(rows[worst])} is off by {diff[worst]:.2e} > {PROBE_TOL:g}"), stats
    return True, f"{msg}; {len(rows)} probe rows exact to {float(diff.max()):.1e}", stats


# ---- the FP32 router layer -------------------------------------------------------------------


def ref_kernel_f32(x_bits: np.ndarray, w_f32: np.ndarray, n: int | None = None) -> np.ndarray:
    """reference.py:72-76 for the router: x @ W[:n].T in FP64, rounded to FP32."""
    x = bf16_to_f32(x_bits).astype(np.float64)
    w = np.asarray(w_f32 if n is None else w_f32[:n], dtype=np.float32).astype(np.float64)
    return (x @ w.T).astype(np.float32)


def split_hi_lo(w_f32: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The router's BF16 hi + lo pair (submission.py:1120-1124): hi = BF16(W), lo = BF16(W - hi),
    both rounded to nearest even; returns their BF16 bits."""
    w = np.asarray(w_f32, dtype=np.float32)
    hi = f32_to_bf16(w)
    lo = f32_to_bf16((w - bf16_to_f32(hi)).astype(np.float32))
    return hi, lo


def check_implementation_f32(x_bits: np.ndarray, w_f32: np.ndarray, out_f32: np.ndarray, n: int | None = None,
                             tol: float = ROUTER_TOL, ref: np.ndarray | None = None) -> tuple[bool, str, dict]:
    """reference.py:84-99 for the router: FP32 ``out_f32`` [M, n] against the FP64 reference
    rounded to FP32 (ROUTER_TOL), then every probe row within PROBE_TOL."""
    if ref is None:
        ref = ref_kernel_f32(x_bits, w_f32, n)
    out = np.asarray(out_f32, dtype=np.float32)
    ok, msg, stats = compare(out, ref, tol)
    rows = probe_rows(x_bits)
    stats["probe_rows"] = int(len(rows))
    if not ok or not len(rows):
        return ok, msg, stats
    d = np.linalg.norm(out[rows].astype(np.float64) - ref[rows].astype(np.float64), axis=-1)
    r = np.maximum(np.linalg.norm(ref[rows].astype(np.float64), axis=-1), 1e-30)
    diff = d / r
    worst = int(diff.argmax())
    stats["probe_worst"] = float(diff[worst])
    if diff[worst] > PROBE_TOL:
        return False, (f"{msg}, but probe row {int(rows[worst])} is off by {diff[worst]:.2e} > {PROBE_TOL:g}"), stats
    return True, f"{msg}; {len(rows)} probe rows exact to {float(diff.max()):.1e}", stats

