"""The tensor-core projection from 12-bit tiles (MUSE_KERNEL_TC_12B) against the FP64 oracle, and
bit for bit against the same kernel reading the BF16 tiles of the original weights
(MUSE_KERNEL_TC_SKINNY) with the same grid: the UMMA sees the same BF16 operands in the same
order, so the two must agree exactly."""

import numpy as np
import pytest
import torch

from muse_bf16_proj_b200 import _lib, codec12, submission
from oracle import contract_ref as O

pytestmark = pytest.mark.gpu


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def to_dev(bits_np: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits_np).view(np.int16)).view(torch.bfloat16).cuda()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _weights(n, k, seed, spice=True):
    """Normal weights with escapes planted: exact zeros, x50 outliers, tiny values, a run of
    escapes at both ends of row 0 (k = 0 and k = K - 1), a row with escapes in every k block, and
    one escape-dense block (more escapes than its area holds)."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randn((n, k), generator=g) * 0.02
    if spice:
        flat = w.view(-1)
        idx = torch.randperm(n * k, generator=g)[: max(8, n * k // 500)]
        flat[idx[0::3]] = 0.0
        flat[idx[1::3]] *= 50.0
        flat[idx[2::3]] = 1e-30
        w[0, :3] = 0.0
        w[0, -3:] = 1e-30
        w[min(n - 1, 5), ::97] = 0.0
        w[8:min(n, 48), 64:128:2] = 0.0  # block (0, 1): up to 40 x 32 escapes
    return bits(w.to(torch.bfloat16))


class _Enc12Tiles:
    def __init__(self, wb):
        n, k = wb.shape
        self.host = codec12.encode(wb)
        self.dev = submission._Enc12Device(self.host, torch.device("cuda"))
        self.tiles = torch.empty(_lib.tiles12_bytes(n, k), dtype=torch.uint8, device="cuda")
        _lib.pack_tiles12(self.dev.view(n), self.tiles.data_ptr(), stream())


def _tiles12_host(enc: codec12.Encoded12) -> np.ndarray:
    """The 12416-byte block layout restated on the host from the row-unit planes and the escape list."""
    n, k = enc.n, enc.k
    units = enc.planes.reshape(n, k // 512, 768)
    lo = units[:, :, :512].reshape(n, k)
    codes = units[:, :, 512:].reshape(n, k // 2)
    rt, nkb = -(-n // 128), k // 64
    out = np.zeros((rt, nkb, 12416), dtype=np.uint8)
    esc = [[] for _ in range(rt * nkb)]  # (r, kk, bits) per block, rows ascending then k
    for row in range(n):
        for v in enc.esc_val[enc.esc_ptr[row]:enc.esc_ptr[row + 1]]:
            kpos = int(v) >> 16
            esc[(row // 128) * nkb + kpos // 64].append((row % 128, kpos % 64, int(v) & 0xFFFF))
    for t in range(rt):
        rows = slice(t * 128, min(n, t * 128 + 128))
        cnt = rows.stop - rows.start
        for b in range(nkb):
            blk_lo = np.zeros((128, 64), np.uint8)
            blk_c = np.zeros((128, 32), np.uint8)
            blk_lo[:cnt] = lo[rows, b * 64:(b + 1) * 64]
            blk_c[:cnt] = codes[rows, b * 32:(b + 1) * 32]
            # slabs: [4][128 rows][16 low bytes], then [2][128 rows][16 code bytes]
            out[t, b, :8192] = blk_lo.reshape(128, 4, 16).transpose(1, 0, 2).reshape(-1)
            out[t, b, 8192:12288] = blk_c.reshape(128, 2, 16).transpose(1, 0, 2).reshape(-1)
            e = esc[t * nkb + b]
            area = np.zeros(32, np.uint32)
            area[0] = (int(enc.bases[t, b // 2]) << 16) | len(e)
            for j, (r, kk, bv) in enumerate(e[:31]):
                area[1 + j] = (r << 22) | (kk << 16) | bv
            out[t, b, 12288:] = area.view(np.uint8)
    return out.reshape(-1)


def _run(enc, x, m, plan, scratch=None):
    n = enc.host.n
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    need = _lib.scratch_bytes(m, n, enc.host.k, plan)
    if need and scratch is None:
        scratch = torch.zeros(need, dtype=torch.uint8, device="cuda")
    _lib.proj_12b_tiles(enc.dev.view(n), enc.tiles.data_ptr(), x.data_ptr(), y.data_ptr(), m, plan, stream(),
                        scratch.data_ptr() if need else 0, need)
    torch.cuda.synchronize()
    assert _lib.device_error(stream()) == 0
    return y


def _skinny_bf16(wb, x, m, tile_n, ctas):
    """The same stream-K kernel on the packed BF16 tiles of the original weights, same tile and grid."""
    n, k = wb.shape
    w = to_dev(wb)
    tiles = torch.empty(_lib.tiles_bytes(n, k), dtype=torch.uint8, device="cuda")
    _lib.pack_tiles(w.data_ptr(), tiles.data_ptr(), n, k, stream())
    plan = _lib.MusePlan(kernel=_lib.KERNEL_TC_SKINNY, tile_n=tile_n, ctas=ctas)
    need = _lib.scratch_bytes(m, n, k, plan)
    scratch = torch.zeros(need, dtype=torch.uint8, device="cuda")
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    _lib.proj_bf16_tiles(x.data_ptr(), tiles.data_ptr(), y.data_ptr(), m, n, k, plan, stream(), scratch.data_ptr(), need)
    torch.cuda.synchronize()
    assert _lib.device_error(stream()) == 0
    return y


def test_pack_tiles12_layout():
    n, k = 200, 1024
    wb = _weights(n, k, 3)
    enc = _Enc12Tiles(wb)
    torch.cuda.synchronize()
    got = enc.tiles.cpu().numpy()
    want = _tiles12_host(enc.host)
    assert np.array_equal(got, want)
    head = want.reshape(-1, 12416)[:, 12288:12292].copy().view(np.uint32) & 0xFFFF
    assert head.max() > 31  # the escape-dense block is covered


@pytest.mark.parametrize("n,k,m,tile_n,ctas,stages,unused", [
    (200, 1024, 3, 16, 7, 3, 1),
    (2304, 8192, 1, 16, 0, 0, 0),
    (2304, 8192, 16, 16, 148, 6, 2),
    (1024, 4096, 33, 64, 100, 3, 3),
    (4096, 8192, 64, 64, 148, 3, 2),
    (1024, 2048, 130, 128, 64, 3, 2),
    (512, 1536, 256, 128, 37, 3, 2),
    (384, 1024, 5, 16, 3, 3, 1),
    (6144, 4096, 7, 16, 296, 6, 2),
    (10240, 8192, 1, 16, 148, 6, 3),
])
def test_tc12_parity(n, k, m, tile_n, ctas, stages, unused):
    wb = _weights(n, k, n + m)
    enc = _Enc12Tiles(wb)
    assert enc.host.n_esc > 0
    xb = bits(torch.randn((m, k), generator=torch.Generator().manual_seed(m)).to(torch.bfloat16))
    x = to_dev(xb)
    plan = _lib.MusePlan(kernel=_lib.KERNEL_TC_12B, tile_n=tile_n, ctas=ctas, stages=stages)
    y = _run(enc, x, m, plan)
    yb = bits(y)
    ok, msg, _ = O.check_implementation(xb, wb, yb)
    assert ok, msg
    rel = O.relative_l2(O.bf16_to_f32(yb), O.bf16_to_f32(O.ref_kernel(xb, wb)))
    assert rel <= 1e-3, rel
    ref = _skinny_bf16(wb, x, m, tile_n, ctas)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), "differs from the kernel on BF16 tiles"


def test_tc12_default_plan_and_repeat():
    n, k, m = 10240, 8192, 1
    wb = _weights(n, k, 11, spice=False)
    enc = _Enc12Tiles(wb)
    xb = bits(torch.randn((m, k), generator=torch.Generator().manual_seed(5)).to(torch.bfloat16))
    x = to_dev(xb)
    plan = _lib.plan_default(m, n, k, weights_12b=True, tiles=True)
    assert plan.kernel == _lib.KERNEL_GEMV_12T
    need = _lib.scratch_bytes(m, n, k, plan)
    scratch = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    y0 = _run(enc, x, m, plan, scratch)
    ok, msg, _ = O.check_implementation(xb, wb, bits(y0))
    assert ok, msg
    for _ in range(3):  # the counters are left at zero: repeated calls give the same bits
        y1 = _run(enc, x, m, plan, scratch)
        assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))


def test_tc12_slice_of_rows():
    """W[:n] of a bigger encoded matrix (the unpooler slice) through the same tiles."""
    n_full, n, k, m = 1024, 384, 2048, 4
    wb = _weights(n_full, k, 21)
    enc = _Enc12Tiles(wb)
    xb = bits(torch.randn((m, k), generator=torch.Generator().manual_seed(9)).to(torch.bfloat16))
    x = to_dev(xb)
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    plan = _lib.MusePlan(kernel=_lib.KERNEL_TC_12B, tile_n=16, ctas=20)
    need = _lib.scratch_bytes(m, n, k, plan)
    scratch = torch.zeros(need, dtype=torch.uint8, device="cuda")
    _lib.proj_12b_tiles(enc.dev.view(n), enc.tiles.data_ptr(), x.data_ptr(), y.data_ptr(), m, plan, stream(),
                        scratch.data_ptr(), need)
    torch.cuda.synchronize()
    ok, msg, _ = O.check_implementation(xb, wb, bits(y), n)
    assert ok, msg


def test_tc12_errors():
    n, k = 256, 1024
    enc = _Enc12Tiles(_weights(n, k, 1))
    x = torch.zeros((4, k), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((4, n), dtype=torch.bfloat16, device="cuda")
    view = enc.dev.view(n)
    with pytest.raises(_lib.MuseError):  # wrong kernel id
        _lib.proj_12b_tiles(view, enc.tiles.data_ptr(), x.data_ptr(), y.data_ptr(), 4,
                            _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE), stream())
    with pytest.raises(_lib.MuseError):  # no scratch
        _lib.proj_12b_tiles(view, enc.tiles.data_ptr(), x.data_ptr(), y.data_ptr(), 4,
                            _lib.MusePlan(kernel=_lib.KERNEL_TC_12B), stream())
    scratch = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    for bad in (_lib.MusePlan(kernel=_lib.KERNEL_TC_12B, tile_n=24), _lib.MusePlan(kernel=_lib.KERNEL_TC_12B, tile_n=256),
                _lib.MusePlan(kernel=_lib.KERNEL_TC_12B, stages=40), _lib.MusePlan(kernel=_lib.KERNEL_TC_12B, stages=1),
                _lib.MusePlan(kernel=_lib.KERNEL_TC_12B, stages=4)):  # not a multiple of the decoder groups
        with pytest.raises(_lib.MuseError):
            _lib.proj_12b_tiles(view, enc.tiles.data_ptr(), x.data_ptr(), y.data_ptr(), 4, bad, stream(),
                                scratch.data_ptr(), scratch.numel())


def test_prepare_reuses_the_12bit_cache(tmp_path):
    """prepare(cache_dir=...) writes the encoding once; a second prepare reads it and serves the
    same bits."""
    import os
    from muse_bf16_proj_b200.dispatch import Dispatch
    n, k, m = 1024, 4096, 4
    wb = _weights(n, k, 77)
    w = to_dev(wb)
    entries = [{"n": n, "k": k, "m_lo": 1, "m_hi": 8, "weights": "12b", "plan": {"kernel": "tc_12b", "tile_n": 16}}]
    xb = bits(torch.randn((m, k), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16))
    x = to_dev(xb)
    outs = []
    for _ in range(2):
        st = submission.prepare({"w": w}, dispatch=Dispatch(entries=entries), encode_12b=True, verbose=False,
                                cache_dir=str(tmp_path))
        outs.append(submission.project(x, st, "w").clone())
    torch.cuda.synchronize()
    assert len(os.listdir(tmp_path)) == 1
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    ok, msg, _ = O.check_implementation(xb, wb, bits(outs[0]))
    assert ok, msg


# ---- the CUDA-core 12-bit GEMV (MUSE_KERNEL_GEMV_12T): decode in registers, M <= 4 ----------------

GEMV12T_CASES = [
    (200, 1024, 3, 0, 0),      # ragged last row tile, the escape-dense block, default grid
    (2304, 8192, 1, 0, 0),
    (2304, 8192, 4, 77, 3),    # row tiles shared by up to 3 CTAs at uneven cuts
    (10240, 8192, 1, 0, 0),    # the 12-bit benchmark shape
    (10240, 8192, 2, 300, 4),
    (384, 1024, 1, 3, 2),      # one CTA a row tile: y written directly
    (1024, 4096, 4, 1000, 3),  # capped at one unit a CTA: 64 contributors a tile
    (6144, 4096, 2, 0, 3),
    (130, 512, 1, 5, 2),       # CTAs spanning two row tiles
]


@pytest.mark.parametrize("n,k,m,ctas,stages", GEMV12T_CASES)
def test_gemv12t_parity(n, k, m, ctas, stages):
    wb = _weights(n, k, 7 * n + m)
    enc = _Enc12Tiles(wb)
    assert enc.host.n_esc > 0
    xb = bits(torch.randn((m, k), generator=torch.Generator().manual_seed(m + 1)).to(torch.bfloat16))
    x = to_dev(xb)
    plan = _lib.MusePlan(kernel=_lib.KERNEL_GEMV_12T, ctas=ctas, stages=stages, flags=_lib.FLAG_PDL)
    y = _run(enc, x, m, plan)
    yb = bits(y)
    ok, msg, _ = O.check_implementation(xb, wb, yb)
    assert ok, msg
    rel = O.relative_l2(O.bf16_to_f32(yb), O.bf16_to_f32(O.ref_kernel(xb, wb)))
    assert rel <= 1e-3, rel
    # Against a torch FP32 product of the original weights (the codec is lossless): FP32 sums in a
    # different order, then one BF16 rounding, so every output is within 2^-8 relative of it.
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = x.float() @ to_dev(wb).float().t()
    err = (y.float() - ref).abs()
    assert bool((err <= ref.abs() * 2.0 ** -8 + 1e-6).all()), float((err / (ref.abs() + 1e-6)).max())
    y2 = _run(enc, x, m, plan)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16)), "not deterministic"


def test_gemv12t_default_plan_and_errors():
    n, k = 1024, 4096
    wb = _weights(n, k, 11)
    enc = _Enc12Tiles(wb)
    for m in (1, 2, 3, 4):
        plan = _lib.plan_default(m, n, k, weights_12b=True, tiles=True)
        assert plan.kernel == _lib.KERNEL_GEMV_12T
    assert _lib.plan_default(5, n, k, weights_12b=True, tiles=True).kernel == _lib.KERNEL_TC_12B
    x = to_dev(bits(torch.randn((5, k)).to(torch.bfloat16)))
    with pytest.raises(_lib.MuseError):  # M = 5 is past the GEMV's token count
        _run(enc, x, 5, _lib.MusePlan(kernel=_lib.KERNEL_GEMV_12T))
    with pytest.raises(_lib.MuseError):  # a ring needs two stages
        _run(enc, x, 1, _lib.MusePlan(kernel=_lib.KERNEL_GEMV_12T, stages=1))
