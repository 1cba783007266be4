"""Parity of the row-window kernel (MUSE_KERNEL_TC_ROWS) with the FP64 oracle.

Each CTA owns a window of W rows over K (no split-K partials), or shares its window's K range with
the other CTAs of a 2- or 4-CTA cluster (DSMEM sum in rank order). Cases cover windows that start
inside a 128-row packed tile and cross into the next (several bulk copies a k block), windows of
unequal height, windows past 256 rows (two UMMAs a k step), ragged N and K, every token tile
height, the output wider than the window's rows at the edge (rows past N never stored), and
determinism. Tolerances as tests/test_gpu_parity.py: the reference's check and relative L2 <= 1e-3
against the FP64 result rounded to BF16.
"""

import pytest
import torch

from muse_bf16_proj_b200 import _lib
from test_gpu_parity import _rand_bits, _run_bf16, assert_parity, stream, to_dev

pytestmark = pytest.mark.gpu


def rows_plan(tile_n=0, split=1, ctas=0, stages=0, pdl=True):
    return _lib.MusePlan(kernel=_lib.KERNEL_TC_ROWS, tile_n=tile_n, split=split, ctas=ctas, stages=stages,
                         flags=_lib.FLAG_PDL if pdl else 0)


CASES = [
    # (n, k, m, split, ctas): the BASELINE decode shapes, the reference's layers, uneven windows
    (6144, 4096, 1, 1, 0), (6144, 4096, 16, 1, 0), (6144, 4096, 32, 1, 0), (6144, 4096, 128, 1, 0),
    (10240, 8192, 1, 1, 0), (10240, 8192, 4, 1, 0),
    (2304, 8192, 1, 2, 0), (2304, 8192, 16, 2, 0), (2304, 8192, 8, 4, 0), (4096, 8192, 16, 2, 0),
    (8192, 1024, 1, 1, 0), (8192, 4096, 32, 1, 0), (1024, 4096, 1, 2, 0),
    (57344, 8192, 1, 1, 148),  # windows of 384 / 400 rows: two UMMAs a k step
    (1000, 1280, 3, 1, 0), (1000, 1280, 5, 2, 0), (200, 200, 7, 1, 0), (136, 4160, 17, 4, 0),
    (6144, 4096, 16, 1, 40), (6144, 4096, 16, 2, 96),
]


@pytest.mark.parametrize("n,k,m,split,ctas", CASES)
def test_rows_parity(n, k, m, split, ctas):
    xb, wb = _rand_bits((m, k), 31 + m + n), _rand_bits((n, k), 47 + n + k, 0.02)
    y = _run_bf16(xb, wb, rows_plan(split=split, ctas=ctas), tiles=True)
    assert_parity(xb, wb, y, what=f"tc_rows n={n} k={k} m={m} split={split} ctas={ctas}")


@pytest.mark.parametrize("tile_n", [16, 32, 64, 128])
def test_rows_token_tiles(tile_n):
    m = min(tile_n, 13)
    xb, wb = _rand_bits((m, 2048), 5 + tile_n), _rand_bits((3000, 2048), 6, 0.02)
    y = _run_bf16(xb, wb, rows_plan(tile_n=tile_n, split=1 if tile_n < 128 else 2), tiles=True)
    assert_parity(xb, wb, y, what=f"tc_rows tile_n={tile_n}")


def test_rows_output_slice_and_determinism():
    """W[:n] of a bigger packed matrix (the unpooler slice) twice, bitwise equal."""
    m, k, big, n = 8, 4096, 8192, 1024
    xb, wb = _rand_bits((m, k), 77), _rand_bits((big, k), 78, 0.02)
    x, w = to_dev(xb), to_dev(wb)
    t = torch.empty(_lib.tiles_bytes(big, k), dtype=torch.uint8, device="cuda")
    _lib.pack_tiles(w.data_ptr(), t.data_ptr(), big, k, stream())
    outs = []
    for split in (1, 2, 1):
        y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        _lib.proj_bf16_tiles(x.data_ptr(), t.data_ptr(), y.data_ptr(), m, n, k, rows_plan(split=split), stream())
        outs.append(y)
    assert_parity(xb, wb[:n], outs[0], what="tc_rows slice")
    assert torch.equal(outs[0], outs[2])
    assert_parity(xb, wb[:n], outs[1], what="tc_rows slice split 2")


def test_rows_graph_replay_with_fresh_inputs():
    """Captured once, replayed with new x copied into the captured buffer (the reference harness)."""
    m, n, k = 16, 6144, 4096
    wb = _rand_bits((n, k), 90, 0.02)
    w = to_dev(wb)
    t = torch.empty(_lib.tiles_bytes(n, k), dtype=torch.uint8, device="cuda")
    _lib.pack_tiles(w.data_ptr(), t.data_ptr(), n, k, stream())
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    plan = rows_plan()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _lib.proj_bf16_tiles(x.data_ptr(), t.data_ptr(), y.data_ptr(), m, n, k, plan,
                             torch.cuda.current_stream().cuda_stream)
    for seed in (91, 92):
        xb = _rand_bits((m, k), seed)
        x.copy_(to_dev(xb))
        g.replay()
        assert_parity(xb, wb, y, what=f"tc_rows graph replay {seed}")


def test_rows_plan_errors():
    with pytest.raises(_lib.MuseError):
        _lib.scratch_bytes(129, 6144, 4096, rows_plan())  # more than 128 tokens
    with pytest.raises(_lib.MuseError):
        _lib.scratch_bytes(16, 6144, 4096, rows_plan(split=3))
    with pytest.raises(_lib.MuseError):
        _lib.scratch_bytes(16, 57344, 8192, rows_plan(ctas=64))  # windows of 896 rows
    assert _lib.scratch_bytes(16, 6144, 4096, rows_plan()) == 0


def _run_rows_packed(xb, wb, plan):
    """The window-major path: muse_pack_rows with the plan's windows, then muse_proj_bf16_rows."""
    x, w = to_dev(xb), to_dev(wb)
    m, k = x.shape
    n = w.shape[0]
    groups = _lib.rows_groups(m, n, k, plan)
    wr = torch.empty(_lib.rows_bytes(n, k, groups), dtype=torch.uint8, device="cuda")
    _lib.pack_rows(w.data_ptr(), wr.data_ptr(), n, k, groups, stream())
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    _lib.proj_bf16_rows(x.data_ptr(), wr.data_ptr(), y.data_ptr(), m, n, k, plan, stream())
    return y


@pytest.mark.parametrize("n,k,m,split,ctas", CASES)
def test_rows_window_major_parity(n, k, m, split, ctas):
    xb, wb = _rand_bits((m, k), 31 + m + n), _rand_bits((n, k), 47 + n + k, 0.02)
    plan = rows_plan(split=split, ctas=ctas)
    y = _run_rows_packed(xb, wb, plan)
    assert_parity(xb, wb, y, what=f"tc_rows window-major n={n} k={k} m={m} split={split} ctas={ctas}")
    # The same windows and K order as the packed-tile source: bit for bit equal.
    y2 = _run_bf16(xb, wb, plan, tiles=True)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)


def test_pack_rows_layout():
    """The window-major copy holds W's bits where the layout puts them (row r of window g, k block kb,
    chunk c at c ^ (r % 8)); rows past N and columns past K are zero."""
    import numpy as np
    n, k, groups = 200, 136, 5
    wb = _rand_bits((n, k), 9, 0.02)
    w = to_dev(wb)
    wr = torch.empty(_lib.rows_bytes(n, k, groups), dtype=torch.uint8, device="cuda")
    _lib.pack_rows(w.data_ptr(), wr.data_ptr(), n, k, groups, stream())
    torch.cuda.synchronize()
    got = wr.cpu().numpy().view(np.uint16)
    units16, nkb = -(-n // 16), -(-k // 64)
    base, extra = units16 // groups, units16 % groups
    padded = np.zeros((units16 * 16, nkb * 64), np.uint16)
    padded[:n, :k] = wb
    expect = np.zeros_like(got)
    for g in range(groups):
        u0 = g * base + min(g, extra)
        length = base + (1 if g < extra else 0)
        rows = 16 * length
        for kb in range(nkb):
            blk = (16 * u0 * nkb * 64 + kb * rows * 64)
            for r in range(rows):
                for c in range(8):
                    dst = blk + r * 64 + (c ^ (r % 8)) * 8
                    expect[dst:dst + 8] = padded[16 * u0 + r, kb * 64 + c * 8:kb * 64 + c * 8 + 8]
    assert np.array_equal(got, expect)
