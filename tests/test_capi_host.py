"""The C ABI without a GPU: the library loads, exports every declared symbol, and rejects bad
arguments with its documented error codes before touching the device."""

import ctypes

import pytest

from muse_bf16_proj_b200 import _lib
from muse_bf16_proj_b200.dispatch import Dispatch


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = _lib.declared_symbols()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    assert _lib.version().startswith("muse_proj_b200")


def test_declared_signatures_are_bound():
    assert set(_lib.declared_symbols()) == set(_lib._SIGNATURES)


def test_proj_argument_errors_before_any_device_work():
    lib = _lib.load()
    plan = _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE, split=1, tile_n=16)
    p = ctypes.byref(plan)
    assert lib.muse_proj_bf16(None, 16, 16, 1, 128, 64, p, None, 0, None) == -1
    assert lib.muse_proj_bf16(16, 16, 16, 0, 128, 64, p, None, 0, None) == -1
    assert lib.muse_proj_bf16(18, 16, 16, 1, 128, 64, p, None, 0, None) == -2   # x misaligned
    assert lib.muse_proj_bf16(16, 16, 16, 1, 128, 60, p, None, 0, None) == -2   # K * 2 not a multiple of 16
    assert lib.muse_proj_bf16(16, 16, 16, 1, 128, 64, None, None, 0, None) == -1
    assert lib.muse_proj_bf16_tiles(None, 16, 16, 1, 128, 64, p, None, 0, None) == -1
    assert lib.muse_proj_bf16_tiles(16, 16, 16, 1, 128, 64, ctypes.byref(_lib.MusePlan(kernel=1)), None, 0, None) == -7
    assert lib.muse_pack_tiles(None, 16, 128, 64, None) == -1
    assert lib.muse_pack_tiles(16, 16, 128, 60, None) == -2
    b = ctypes.c_int64()
    assert lib.muse_tiles_bytes(200, 200, ctypes.byref(b)) == 0 and b.value == 2 * 4 * 16384
    enc = _lib.MuseEnc12(16, 16, 16, 16, 128, 512, 0)
    plan12 = _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE)
    assert lib.muse_proj_12b(ctypes.byref(enc), 16, 16, 1, ctypes.byref(plan12), None) == -7
    enc_bad = _lib.MuseEnc12(None, 16, 16, 16, 128, 512, 0)
    assert lib.muse_proj_12b(ctypes.byref(enc_bad), 16, 16, 1, ctypes.byref(plan12), None) == -1
    assert b"null" in lib.muse_last_error()
    # 12-bit tiles: sizes, K rules, null and plan checks
    assert lib.muse_tiles12_bytes(200, 1024, ctypes.byref(b)) == 0 and b.value == 2 * 16 * 12416
    assert lib.muse_tiles12_bytes(200, 1000, ctypes.byref(b)) == -3
    assert lib.muse_pack_tiles12(ctypes.byref(enc_bad), 16, None) == -1
    assert lib.muse_pack_tiles12(ctypes.byref(enc), 18, None) == -2
    t12 = _lib.MusePlan(kernel=_lib.KERNEL_TC_12B)
    assert lib.muse_proj_12b_tiles(ctypes.byref(enc), None, 16, 16, 1, ctypes.byref(t12), None, 0, None) == -1
    assert lib.muse_proj_12b_tiles(ctypes.byref(enc), 16, 18, 16, 1, ctypes.byref(t12), None, 0, None) == -2
    assert lib.muse_proj_12b_tiles(ctypes.byref(enc), 16, 16, 16, 1, ctypes.byref(plan12), None, 0, None) == -7
    # FP32 router: sizes, K rule, null / alignment / plan checks before any device work
    assert lib.muse_router_tiles_bytes(256, 8192, ctypes.byref(b)) == 0 and b.value == 2 * 256 * 16384
    assert lib.muse_router_tiles_bytes(256, 100, ctypes.byref(b)) == -3
    assert lib.muse_pack_router(None, 16, 256, 8192, None) == -1
    assert lib.muse_pack_router(20, 16, 256, 8192, None) == -2
    f32 = _lib.MusePlan(kernel=_lib.KERNEL_F32_GEMV)
    assert lib.muse_proj_f32(16, None, 16, 16, 1, 256, 8192, ctypes.byref(f32), None, 0, None) == -1  # FP32 path needs W
    assert lib.muse_proj_f32(16, 16, 16, 16, 33, 256, 8192, ctypes.byref(f32), None, 0, None) == -3   # M <= 32
    assert lib.muse_proj_f32(18, 16, 16, 16, 1, 256, 8192, ctypes.byref(f32), None, 0, None) == -2
    tc = _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE)
    assert lib.muse_proj_f32(16, 16, None, 16, 16, 256, 8192, ctypes.byref(tc), None, 0, None) == -1  # needs tiles
    assert lib.muse_proj_f32(16, 16, 16, 16, 16, 256, 8192, ctypes.byref(_lib.MusePlan(kernel=5)), None, 0, None) == -7


def test_plan_default_without_device():
    p = _lib.plan_default(1, 6144, 4096)
    assert p.kernel == _lib.KERNEL_GEMV_BF16
    p = _lib.plan_default(1, 6144, 4096, tiles=True)
    assert p.kernel == _lib.KERNEL_GEMV_TILES and p.chunk == 8 and p.warps == 4
    p = _lib.plan_default(3, 6144, 4096, tiles=True)
    assert p.kernel == _lib.KERNEL_TC_STREAMK and p.tile_n == 16
    p = _lib.plan_default(2, 6144, 1 << 20, tiles=True)  # x past the GEMV's shared memory: stream-K
    assert p.kernel == _lib.KERNEL_TC_STREAMK
    p = _lib.plan_default(16, 6144, 4096)
    assert p.kernel == _lib.KERNEL_TC_TILE and p.tile_n == 16 and 1 <= p.split <= 8
    p = _lib.plan_default(200, 6144, 4096, tiles=True)
    assert p.kernel == _lib.KERNEL_TC_TILE and p.tile_n == 256
    p = _lib.plan_default(4096, 10240, 8192, tiles=True)
    assert p.kernel == _lib.KERNEL_TC_GEMM2
    with pytest.raises(_lib.MuseError):
        _lib.plan_default(4096, 10240, 8192)  # needs packed tiles
    p = _lib.plan_default(1, 10240, 8192, weights_12b=True)
    assert p.kernel == _lib.KERNEL_GEMV_12B
    p = _lib.plan_default(1, 10240, 8192, weights_12b=True, tiles=True)
    assert p.kernel == _lib.KERNEL_GEMV_12T and p.stages == 3
    p = _lib.plan_default(16, 10240, 8192, weights_12b=True, tiles=True)
    assert p.kernel == _lib.KERNEL_TC_12B and p.tile_n == 16 and p.ctas > 0
    p = _lib.plan_default(300, 2304, 8192, weights_12b=True, tiles=True)
    assert p.kernel == _lib.KERNEL_TC_12B and p.tile_n == 128
    with pytest.raises(_lib.MuseError):
        _lib.plan_default(1, 2304, 1000, weights_12b=True, tiles=True)
    p = _lib.plan_default(2, 256, 8192, f32=True)
    assert p.kernel == _lib.KERNEL_F32_GEMV
    assert _lib.plan_default(16, 256, 8192, f32=True).kernel == _lib.KERNEL_F32_GEMV
    p = _lib.plan_default(17, 256, 8192, f32=True)
    assert p.kernel == _lib.KERNEL_TC_TILE and p.tile_n == 16 and p.split == 16 and p.flags & _lib.FLAG_GLOBAL_SPLIT
    p = _lib.plan_default(256, 256, 8192, f32=True)
    assert p.split == 8
    with pytest.raises(_lib.MuseError):
        _lib.plan_default(0, 10, 10)


def test_dispatch_table_lookup_and_defaults():
    entries = [
        {"n": 6144, "k": 4096, "m_lo": 1, "m_hi": 1, "weights": "12b", "plan": {"kernel": "gemv_12b", "warps": 8}},
        {"n": 6144, "k": 4096, "m_lo": 1, "m_hi": 4, "weights": "bf16", "plan": {"kernel": "gemv_bf16", "warps": 16}},
        {"n": 6144, "k": 4096, "m_lo": 5, "m_hi": 32, "plan": {"kernel": "tc_tile", "tile_n": 32, "split": 3}},
    ]
    d = Dispatch(entries=entries)
    plan, fmt = d.plan(1, 6144, 4096, have_12b=True)
    assert fmt == "12b" and plan.kernel == _lib.KERNEL_GEMV_12B
    plan, fmt = d.plan(1, 6144, 4096, have_12b=False)
    assert fmt == "bf16" and plan.kernel == _lib.KERNEL_GEMV_BF16 and plan.warps == 16
    plan, fmt = d.plan(17, 6144, 4096)
    assert plan.kernel == _lib.KERNEL_TC_TILE and plan.split == 3 and plan.tile_n == 32
    plan, fmt = d.plan(64, 6144, 4096)   # no row: library default (packed tiles)
    assert plan.kernel == _lib.KERNEL_TC_STREAMK and plan.tile_n == 64
    plan, fmt = d.plan(64, 6144, 4096, tiles=False)
    assert plan.kernel == _lib.KERNEL_TC_TILE and plan.tile_n == 64
    assert d.wants_12b(6144, 4096) and not d.wants_12b(6144, 8192)
    assert _lib.MusePlan.from_dict(plan.as_dict()).key() == plan.key()


def test_committed_table_rows_are_valid():
    d = Dispatch()
    for e in d.entries:
        p = _lib.MusePlan.from_dict(e["plan"])
        assert p.kernel in _lib.KERNEL_NAMES
        assert e["m_lo"] <= e["m_hi"]
        if p.kernel == _lib.KERNEL_GEMV_12B:
            assert e["weights"] == "12b"


def test_gather_argument_errors():
    """The fused all-gather entry point validates its descriptor before touching the GPU."""
    assert _lib.peer_ctl_bytes() == 384
    gat = _lib.MuseGather()
    gat.world, gat.rank, gat.ldy, gat.col0 = 2, 2, 64, 0
    plan = _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE, tile_n=16, split=1)

    def code():
        with pytest.raises(_lib.MuseError) as e:
            _lib.proj_bf16_tiles_gather(16, 16, 1, 64, 64, gat, plan, 0)
        return e.value.code

    assert code() == -1  # rank >= world
    gat.rank, gat.col0 = 1, 8
    assert code() == -3  # columns col0 .. col0 + n past ldy
    gat.col0, gat.world = 0, 9
    assert code() == -1  # more ranks than MUSE_MAX_PEERS
    gat.world = 2
    assert code() == -1  # null buffers
    gat.y[0] = gat.y[1] = gat.ctl[0] = gat.ctl[1] = 256
    gat.ldy = 68
    assert code() == -3  # ldy not a multiple of 8
    gat.ldy = 64
    plan.kernel = _lib.KERNEL_TC_STREAMK
    assert code() == -7  # the fused epilogue lives in the tile kernel and the pair GEMM only
    plan.kernel, plan.split = _lib.KERNEL_TC_TILE, 4
    assert code() == -7  # a cluster K split is refused (scratch split only)
    with pytest.raises(_lib.MuseError):
        _lib.ipc_export(0)
    with pytest.raises(ValueError):
        _lib.ipc_open(b"short", 0)


def test_stream_k_scratch_sizing_and_plan_errors():
    """Scratch sizing of the stream-K plans (12-bit GEMV, pair GEMM) and their argument checks,
    before any device work."""
    g12 = _lib.MusePlan(kernel=_lib.KERNEL_GEMV_12T)
    need = _lib.scratch_bytes(1, 10240, 8192, g12)
    assert need >= 65536 and need % 4 == 0  # tickets, then FP32 partials of shared row tiles
    assert _lib.scratch_bytes(4, 10240, 8192, g12) > need  # partials scale with the token tile
    with pytest.raises(_lib.MuseError) as e:  # one to four tokens
        _lib.scratch_bytes(5, 10240, 8192, g12)
    assert e.value.code == -3
    with pytest.raises(_lib.MuseError) as e:  # a ring needs two stages
        _lib.scratch_bytes(1, 10240, 8192, _lib.MusePlan(kernel=_lib.KERNEL_GEMV_12T, stages=1))
    assert e.value.code == -7
    sk = _lib.MusePlan(kernel=_lib.KERNEL_TC_GEMM2, flags=_lib.FLAG_STREAMK)
    need = _lib.scratch_bytes(256, 10240, 8192, sk)
    assert need > 65536 and (need - 65536) % (2 * 128 * 256 * 4) == 0  # whole 128 KB tile halves
    assert _lib.scratch_bytes(256, 10240, 8192, _lib.MusePlan(kernel=_lib.KERNEL_TC_GEMM2)) == 0
    tail = _lib.MusePlan(kernel=_lib.KERNEL_TC_GEMM2, flags=_lib.FLAG_SK_TAIL)
    need = _lib.scratch_bytes(8192, 7168, 8192, tail)  # 896 tiles: a tail after the whole waves
    assert need > 65536 and (need - 65536) % (2 * 128 * 256 * 4) == 0
    assert need < _lib.scratch_bytes(8192, 7168, 8192, sk)  # only the tail's tiles have partials


def test_pair_kernel_plans_and_scratch():
    """The medium-M pair kernel's plan checks and scratch sizes, on the host (no device work)."""
    pk = lambda **kw: _lib.MusePlan(kernel=_lib.KERNEL_TC_PAIRK, **kw)
    # No split: no scratch. A split: 64 KB of counters, then [tiles][2][split][tile_n][128] FP32.
    assert _lib.scratch_bytes(256, 2304, 8192, pk(tile_n=256, split=1)) == 0
    assert _lib.scratch_bytes(256, 2304, 8192, pk(tile_n=256, split=8)) == 65536 + 9 * 2 * 8 * 256 * 128 * 4
    for bad in (pk(tile_n=24), pk(tile_n=272),                  # tile_n a multiple of 16 up to 256;
                pk(tile_n=256, split=3), pk(tile_n=16, split=32)):  # the split divides tile_n...
        with pytest.raises(_lib.MuseError) as e:
            _lib.scratch_bytes(256, 2304, 8192, bad)
        assert e.value.code == -7
    with pytest.raises(_lib.MuseError):  # ... and does not exceed the k blocks (K = 1024: 16)
        _lib.scratch_bytes(256, 2304, 1024, pk(tile_n=256, split=32))
    # Stream-K: runs of at most one tile, partials for every tile sized for the most contributors.
    sk = pk(tile_n=256, flags=_lib.FLAG_STREAMK)
    need = _lib.scratch_bytes(256, 10240, 8192, sk)
    assert need > 65536 and (need - 65536) % (2 * 256 * 128 * 4) == 0
    with pytest.raises(_lib.MuseError, match="exceed a tile"):  # 448 tiles for 74 pairs
        _lib.scratch_bytes(512, 57344, 8192, sk)


def test_tile_gemv_plan_checks():
    """The decode tile GEMV needs no scratch and refuses plans it cannot run, on the host."""
    gt = lambda **kw: _lib.MusePlan(kernel=_lib.KERNEL_GEMV_TILES, **kw)
    for m in (1, 2, 3, 4):
        assert _lib.scratch_bytes(m, 6144, 4096, gt()) == 0
    assert _lib.scratch_bytes(1, 6144, 4096, gt(warps=16, split=16)) == 0
    assert _lib.scratch_bytes(1, 130, 136, gt(warps=4, split=2)) == 0
    assert _lib.scratch_bytes(4, 6144, 4096, gt(warps=16, split=4, chunk=4)) == 0
    assert _lib.scratch_bytes(2, 6144, 4096, gt(warps=8, split=4, chunk=8)) == 0
    for m, n, k, plan, code in ((5, 6144, 4096, gt(), -3),                     # at most 4 tokens
                                (1, 6144, 4096, gt(warps=8, split=3), -7),     # split divides the warps
                                (1, 6144, 4096, gt(warps=17), -7),             # at most 16 warps
                                (1, 6144, 4096, gt(chunk=3), -7),              # 1, 2, 4 or 8 quads a warp
                                (3, 6144, 4096, gt(chunk=8), -7),              # 8 only for M <= 2
                                (1, 6144, 128, gt(warps=8, split=4), -7),      # split <= k blocks (2)
                                (4, 6144, 1 << 16, gt(), -3)):                  # x must fit shared memory
        with pytest.raises(_lib.MuseError) as e:
            _lib.scratch_bytes(m, n, k, plan)
        assert e.value.code == code, (m, n, k, plan.as_dict())


def test_device_encoder_argument_errors():
    """muse_encode12_device / _escapes reject bad shapes, null or misaligned pointers before any launch."""
    lib = _lib.load()
    enc, esc = lib.muse_encode12_device, lib.muse_encode12_device_escapes
    assert enc(None, 128, 512, 16, 16, 16, None) == -1            # null W
    assert enc(16, 0, 512, 16, 16, 16, None) == -1                # N < 1
    assert enc(16, 128, 256, 16, 16, 16, None) == -1              # K < 512
    assert enc(16, 128, 1000, 16, 16, 16, None) == -3             # K % 512
    assert enc(16, 128, 65536 + 512, 16, 16, 16, None) == -3      # K > 65536
    assert enc(16, 1 << 20, 4096, 16, 16, 16, None) == -3         # N * K >= 2^31
    assert b"2^31" in lib.muse_last_error()
    assert enc(18, 128, 512, 16, 16, 16, None) == -2              # W not 16-byte aligned
    assert enc(16, 128, 512, 12, 16, 16, None) == -2              # planes not 8-byte aligned
    assert enc(16, 128, 512, None, 16, 16, None) == -1
    assert esc(16, 128, 512, None, 16, 16, 8, None) == -1         # null bases
    assert esc(16, 128, 512, 16, 16, None, 8, None) == -1         # escapes expected, no buffer
    assert esc(16, 128, 512, 16, 16, 16, -1, None) == -1          # negative capacity
    assert esc(16, 128, 1000, 16, 16, 16, 8, None) == -3


def test_library_exports_nothing_undeclared():
    """Every muse_* symbol the library exports is declared in include/muse_proj.h (the ABI is the
    header, nothing beside it)."""
    import shutil
    import subprocess

    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("no nm")
    out = subprocess.run([nm, "-D", "--defined-only", _lib.LIB], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.split() and line.split()[-1].startswith("muse_")}
    assert exported == set(_lib.declared_symbols())
