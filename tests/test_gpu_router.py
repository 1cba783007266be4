"""The FP32 router (reference.py:20-29, submission.py:1027-1076) on this build's kernels: the hi | lo
tile packing bit for bit against the oracle's split, both plans (FP32 on CUDA cores, hi + lo on the
tensor cores) against the FP64 oracle at the router tolerance (relative L2 1e-4, probe rows 1e-3),
the reference's router cases through kernel_fn, determinism and graph replay."""

import numpy as np
import pytest
import torch

from muse_bf16_proj_b200 import _lib, submission
from muse_bf16_proj_b200 import contract as C
from oracle import contract_ref as O

pytestmark = pytest.mark.gpu


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


@pytest.fixture(scope="module")
def router_w():
    return C.generate_weights(C.WEIGHTS_SEED, device="cpu")["router"]


@pytest.fixture(scope="module")
def state(router_w):
    return submission.prepare({"router": router_w.cuda()}, verbose=False)


def _untile(tiles: np.ndarray, n: int, k2: int) -> np.ndarray:
    """Packed tiles (muse_pack_tiles layout) back to the [n, k2] BF16 bits they hold."""
    nkb = k2 // 64
    t = tiles.view(np.uint16).reshape(-1, nkb, 128, 8, 8)  # [rt, kb, row, chunk position, 8]
    out = np.zeros((t.shape[0] * 128, k2), np.uint16)
    for r in range(128):
        for pos in range(8):
            c = pos ^ (r % 8)
            for kb in range(nkb):
                out[np.arange(t.shape[0]) * 128 + r, kb * 64 + c * 8: kb * 64 + c * 8 + 8] = t[:, kb, r, pos, :]
    return out[:n]


def test_pack_router_matches_oracle_split():
    g = torch.Generator().manual_seed(3)
    n, k = 200, 256
    w = torch.randn((n, k), generator=g) * 0.01
    w[0, :5] = torch.tensor([0.0, -0.0, 1e-40, 3.0e38, -1.5])
    wd = w.cuda()
    tiles = torch.empty(_lib.router_tiles_bytes(n, k), dtype=torch.uint8, device="cuda")
    _lib.pack_router(wd.data_ptr(), tiles.data_ptr(), n, k, stream())
    torch.cuda.synchronize()
    got = _untile(tiles.cpu().numpy(), n, 2 * k)
    hi, lo = O.split_hi_lo(w.numpy())
    assert np.array_equal(got[:, :k], hi)
    assert np.array_equal(got[:, k:], lo)


def _run(state, xb, plan):
    w = state["fp32"]["router"]
    m, k = xb.shape
    n = w.shape[0]
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    need = _lib.scratch_bytes(m, n, k, plan)
    scratch = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    _lib.proj_f32(x.data_ptr(), w.data_ptr(), state["fp32_tiles"]["router"].data_ptr(), y.data_ptr(), m, n, k, plan,
                  stream(), scratch.data_ptr() if need else 0, need)
    torch.cuda.synchronize()
    assert _lib.device_error(stream()) == 0
    if need:
        assert int(torch.count_nonzero(scratch[: 64 * 1024])) == 0
    return y.cpu().numpy()


PLANS = [
    ("f32", 1, {}), ("f32", 2, {}), ("f32", 3, {}), ("f32", 8, {}), ("f32", 9, {}), ("f32", 16, {}), ("f32", 32, {}),
    ("tc", 1, {"tile_n": 16, "split": 32, "flags": 1}), ("tc", 8, {"tile_n": 16, "split": 16, "flags": 1}),
    ("tc", 9, {"tile_n": 16, "split": 8, "flags": 1}), ("tc", 33, {"tile_n": 64, "split": 12, "flags": 1}),
    ("tc", 130, {"tile_n": 128, "split": 4, "flags": 1}), ("tc", 300, {"tile_n": 256, "split": 2, "flags": 1}),
    ("tc", 64, {"tile_n": 64, "split": 1}),
]


@pytest.mark.parametrize("kind,m,extra", PLANS)
def test_router_plans(state, router_w, kind, m, extra):
    data = C.generate_input(m, "router", 6000 + m, "outliers" if m % 2 else "normal", device="cpu")
    xb = bits(data["x"])
    kernel = _lib.KERNEL_F32_GEMV if kind == "f32" else _lib.KERNEL_TC_TILE
    plan = _lib.MusePlan.from_dict({"kernel": kernel, **extra})
    y = _run(state, xb, plan)
    ok, msg, stats = O.check_implementation_f32(xb, router_w.numpy(), y)
    assert ok, f"{kind} m={m}: {msg}"
    if kind == "f32":  # FP32 weights, FP32 accumulation: far inside the tolerance
        assert stats["rel_l2"] < 1e-6, stats
    y2 = _run(state, xb, plan)
    assert np.array_equal(y, y2), "not deterministic"


@pytest.mark.parametrize("m,seed,dist", [(8, 7008, "normal"), (9, 7009, "outliers"), (1, 8001, "normal"),
                                         (16, 8016, "normal"), (32, 8032, "normal"), (128, 8128, "normal"),
                                         (256, 8256, "normal"), (1000, 4242, "normal")])
def test_router_reference_cases_through_kernel_fn(state, router_w, m, seed, dist):
    data = C.generate_input(m, "router", seed, dist, device="cpu")
    y = submission.kernel_fn({"x": data["x"].cuda(), "config": data["config"]}, state)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32 and y.shape == (m, 256)
    ok, msg, _ = O.check_implementation_f32(bits(data["x"]), router_w.numpy(), y.cpu().numpy())
    assert ok, f"router m={m}: {msg}"


def test_router_graph_replay(state, router_w):
    for m in (4, 24):
        xs = [C.generate_input(m, "router", 500 + m + i, "normal", device="cpu")["x"] for i in range(3)]
        x = xs[0].cuda()
        cfg = {"m": m, "n": 256, "k": 8192, "layer": "router"}
        submission.kernel_fn({"x": x, "config": cfg}, state)  # first call outside capture (scratch)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            y = submission.kernel_fn({"x": x, "config": cfg}, state)
        for xi in xs:
            x.copy_(xi.cuda())
            g.replay()
            torch.cuda.synchronize()
            ok, msg, _ = O.check_implementation_f32(bits(xi), router_w.numpy(), y.cpu().numpy())
            assert ok, f"replay m={m}: {msg}"
        del g
