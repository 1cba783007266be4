"""Parity of the medium-M pair GEMM (MUSE_KERNEL_TC_PAIRK: 256 W rows x tile_n tokens a CTA pair, W as
the UMMA A operand, K split across pairs that reduce it together) with the FP64 oracle.

Cases: the reference's medium-M shapes (qkv_gate, pooler, unpooler, o at 64..256 tokens) with 8-way
splits; ragged M, N and K with uneven K ranges (the tensor store clipping the edges); N not a multiple of 8 (plain
stores); several token tiles; no split
with more pairs than fit at once (several waves); tile_n 16 with 16 splits; two-stage rings; the
counters back at zero after every launch; determinism; programmatic launches back to back; the host's
refusal of a split grid that cannot be resident at once. Tolerances as tests/test_gpu_parity.py.
"""

import numpy as np
import pytest
import torch

from muse_bf16_proj_b200 import _lib
from test_gpu_parity import _rand_bits, _run_bf16, assert_parity, bits, scratch_buf, stream, to_dev

pytestmark = pytest.mark.gpu


def pk_plan(t=0, s=0, stages=0, flags=0):
    return _lib.MusePlan(kernel=_lib.KERNEL_TC_PAIRK, tile_n=t, split=s, stages=stages, flags=flags)


CASES = [
    # (m, n, k, tile_n, split, stages)
    (256, 2304, 8192, 256, 8, 0),   # qkv_gate, M = 256: 9 tiles x 8 = 72 pairs
    (128, 2304, 8192, 128, 8, 0),   # qkv_gate, M = 128
    (64, 2304, 8192, 64, 8, 0),     # qkv_gate, M = 64
    (256, 4096, 8192, 256, 4, 0),   # pooler
    (256, 8192, 4096, 256, 2, 0),   # unpooler
    (128, 8192, 1024, 128, 2, 0),   # o
    (200, 1000, 640, 208, 4, 0),    # ragged: 10 k blocks as 2 + 3 + 2 + 3, token slices of 52; y stores clipped
    (100, 3000, 4160, 112, 4, 2),   # ragged, two stages
    (64, 1001, 1024, 64, 2, 0),     # N not a multiple of 8: plain stores instead of the tensor store
    (300, 4096, 1024, 160, 1, 0),   # two token tiles, no split
    (512, 28672, 1024, 256, 1, 0),  # no split, 224 pairs: several waves
    (16, 4096, 8192, 16, 4, 0),     # the smallest tile
    (33, 2304, 8192, 48, 6, 3),     # odd M, 6 splits of 128 k blocks
]


@pytest.mark.parametrize("m,n,k,t,s,stages", CASES)
def test_pairk_parity(m, n, k, t, s, stages):
    xb, wb = _rand_bits((m, k), 31 + m + k), _rand_bits((n, k), 37 + n, 0.02)
    y = _run_bf16(xb, wb, pk_plan(t, s, stages), tiles=True)
    torch.cuda.synchronize()
    assert _lib.device_error(stream()) == 0
    assert_parity(xb, wb, y, what=f"tc_pairk m={m} n={n} k={k} tile_n={t} split={s} stages={stages}")
    # Every launch leaves its counters at zero (the next launch and other kernels share the scratch).
    assert int(scratch_buf()[:65536].count_nonzero()) == 0


def test_pairk_deterministic():
    m, n, k = 256, 2304, 8192
    xb, wb = _rand_bits((m, k), 3), _rand_bits((n, k), 4, 0.02)
    y1 = bits(_run_bf16(xb, wb, pk_plan(256, 8), tiles=True))
    y2 = bits(_run_bf16(xb, wb, pk_plan(256, 8), tiles=True))
    assert np.array_equal(y1, y2)


def test_pairk_programmatic_chain():
    """Three programmatic launches back to back on one stream, each on its own inputs, sharing the
    scratch: each output matches the oracle."""
    m, n, k = 128, 2304, 8192
    xs = [_rand_bits((m, k), 50 + i) for i in range(3)]
    wb = _rand_bits((n, k), 60, 0.02)
    w = to_dev(wb)
    t = torch.empty(_lib.tiles_bytes(n, k), dtype=torch.uint8, device="cuda")
    _lib.pack_tiles(w.data_ptr(), t.data_ptr(), n, k, stream())
    sc = scratch_buf()
    outs = []
    for xb in xs:
        x = to_dev(xb)
        y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        _lib.proj_bf16_tiles(x.data_ptr(), t.data_ptr(), y.data_ptr(), m, n, k, pk_plan(128, 8, 0, _lib.FLAG_PDL), stream(),
                             sc.data_ptr(), sc.numel())
        outs.append((x, y))
    torch.cuda.synchronize()
    assert _lib.device_error(stream()) == 0
    for xb, (_, y) in zip(xs, outs):
        assert_parity(xb, wb, y, what="tc_pairk programmatic chain")


def test_pairk_refuses_split_grid_beyond_one_wave():
    m, n, k = 256, 57344, 8192  # 224 row pairs x 2 splits: more pairs than can be resident
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    t = torch.zeros(_lib.tiles_bytes(n, k), dtype=torch.uint8, device="cuda")
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    need = _lib.scratch_bytes(m, n, k, pk_plan(256, 2))
    big = torch.zeros(need, dtype=torch.uint8, device="cuda")
    with pytest.raises(_lib.MuseError, match="resident"):
        _lib.proj_bf16_tiles(x.data_ptr(), t.data_ptr(), y.data_ptr(), m, n, k, pk_plan(256, 2), stream(), big.data_ptr(),
                             big.numel())


SK_CASES = [
    # (m, n, k, tile_n, ctas): the stream-K schedule (equal runs of (tile, k block) units, one a pair)
    (256, 10240, 8192, 256, 0),   # 40 tiles for 74 pairs: runs of 69 of a tile's 128 k blocks
    (128, 6144, 4096, 128, 0),    # 24 tiles
    (256, 2304, 8192, 256, 0),    # 9 tiles: about 9 contributors a tile
    (256, 8192, 1024, 128, 0),    # two token tiles, runs of 13-14 of 16 k blocks
    (200, 1000, 640, 208, 40),    # ragged, 20 pairs; the tensor store clips the edges
    (100, 3000, 4160, 112, 60),   # ragged K, 30 pairs
    (64, 1001, 1024, 64, 20),     # N not a multiple of 8: plain stores
    (33, 2304, 8192, 48, 0),      # 48 tokens in 16-token slices: some contributors reduce nothing
]


@pytest.mark.parametrize("m,n,k,t,ctas", SK_CASES)
def test_pairk_streamk_parity(m, n, k, t, ctas):
    xb, wb = _rand_bits((m, k), 41 + m + k), _rand_bits((n, k), 43 + n, 0.02)
    plan = _lib.MusePlan(kernel=_lib.KERNEL_TC_PAIRK, tile_n=t, ctas=ctas, flags=_lib.FLAG_STREAMK)
    y = _run_bf16(xb, wb, plan, tiles=True)
    torch.cuda.synchronize()
    assert _lib.device_error(stream()) == 0
    assert_parity(xb, wb, y, what=f"tc_pairk stream-K m={m} n={n} k={k} tile_n={t} ctas={ctas}")
    assert int(scratch_buf()[:65536].count_nonzero()) == 0
    again = _run_bf16(xb, wb, plan, tiles=True)  # deterministic: the same grid sums in the same order
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), again.view(torch.int16))


def test_pairk_streamk_refuses_runs_longer_than_a_tile():
    m, n, k = 512, 57344, 8192  # 448 tiles of 128 k blocks for 74 pairs
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    t = torch.zeros(_lib.tiles_bytes(n, k), dtype=torch.uint8, device="cuda")
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    plan = _lib.MusePlan(kernel=_lib.KERNEL_TC_PAIRK, tile_n=256, flags=_lib.FLAG_STREAMK)
    with pytest.raises(_lib.MuseError, match="exceed a tile"):
        _lib.proj_bf16_tiles(x.data_ptr(), t.data_ptr(), y.data_ptr(), m, n, k, plan, stream(), 0, 0)
