"""Host replay of the decode tile GEMV's index arithmetic (csrc/gemv_tiles.cuh) on the packed-tile
layout that muse_pack_tiles writes (tests/test_gpu_parity.py::test_pack_tiles_layout checks the
packer against the same layout on a GPU): row r of a 128-row tile, 16-byte chunk c at position
c ^ (r % 8), tiles [rt][kb] of 16 KB.

For every quad width (QW = 1, 2, 4, 8), quad group, lane and k block, the byte address the kernel
loads and the x chunk it pairs the loaded weights with must name the same W row and k range, and
every (row, k) of W must be covered exactly once. No device work."""

import numpy as np
import pytest


def pack_tiles(w: np.ndarray) -> np.ndarray:
    """The packed layout as bytes: [rt][kb][128 rows][8 positions][8 BF16], zero padded."""
    n, k = w.shape
    rt, nkb = -(-n // 128), -(-k // 64)
    pad = np.zeros((rt * 128, nkb * 64), dtype=np.uint16)
    pad[:n, :k] = w
    t = pad.reshape(rt, 128, nkb, 8, 8).transpose(0, 2, 1, 3, 4).copy()  # [rt][kb][r][c][8]
    out = np.empty_like(t)
    for r in range(128):
        for c in range(8):
            out[:, :, r, c ^ (r % 8)] = t[:, :, r, c]
    return out.reshape(-1).view(np.uint8)


@pytest.mark.parametrize("qw", [1, 2, 4, 8])
def test_lane_addresses_match_rows_and_chunks(qw):
    n, k = 300, 320  # ragged: 3 row tiles, 5 k blocks (the last one padded)
    rng = np.random.default_rng(qw)
    w = rng.integers(1, 1 << 15, size=(n, k), dtype=np.uint16)
    tiles = pack_tiles(w)
    rt, nkb = -(-n // 128), -(-k // 64)
    quads = rt * 32
    seen = np.zeros((rt * 128, nkb * 64), dtype=np.int32)
    for q0 in range(0, quads, qw):  # a warp's first quad: QW-aligned, so its quads share a row tile
        par0 = q0 & 1
        for kb in range(nkb):
            for lane in range(32):
                r4, pos = lane >> 3, lane & 7
                for j in range(qw):
                    # The kernel's load address (gt_load) and x chunk (xe for even quads, xo for odd).
                    addr = ((q0 >> 5) * nkb + kb) * 16384 + (q0 & 31) * 512 + j * 512 + lane * 16
                    par = par0 ^ (j & 1)
                    chunk = pos ^ ((par << 2) | r4)
                    got = tiles[addr:addr + 16].view(np.uint16)
                    row = (q0 + j) * 4 + r4
                    k0 = kb * 64 + chunk * 8
                    assert (q0 + j) >> 5 == q0 >> 5
                    expect = np.zeros(8, dtype=np.uint16)
                    if row < n:
                        valid = max(0, min(8, k - k0))
                        expect[:valid] = w[row, k0:k0 + valid]
                    assert np.array_equal(got, expect), (qw, q0, kb, lane, j)
                    seen[row, k0:k0 + 8] += 1
    assert (seen == 1).all()


def test_segments_cover_k_once():
    """split K segments of a quad: [s nkb / split, (s + 1) nkb / split) tile K exactly."""
    for nkb in (1, 5, 16, 64, 128):
        for split in (1, 2, 4, 8, 16):
            if split > nkb:
                continue
            cover = []
            for s in range(split):
                kb0 = s * nkb // split
                nb = (s + 1) * nkb // split - kb0
                assert nb >= 1
                cover += list(range(kb0, kb0 + nb))
            assert cover == list(range(nkb))
