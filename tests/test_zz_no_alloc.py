"""The no-allocation entry point, muse_proj_bf16_tiles_noalloc.

Some callers cannot allocate device memory: an inference engine's plugin, for instance, is handed
its input and output buffers from the engine's own pool and may not cudaMalloc behind the engine's
back. For them the library keeps the stream-K kernel's split-K scratch in a fixed built-in area
(8 MiB) instead of a caller buffer. These tests call it through the C ABI and check it against the
caller-scratch entry point (muse_proj_bf16_tiles) on two calls in a row, and that a shape needing
more scratch than the area holds is refused. The file is named to be collected last.
"""

import numpy as np
import pytest
import torch

from muse_bf16_proj_b200 import _lib
from oracle import contract_ref as O

pytestmark = pytest.mark.gpu

TIGHT_REL_L2 = 1e-3  # the parity tests' bound against the FP64 reference


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _packed(w: torch.Tensor, stream: int) -> torch.Tensor:
    n, k = w.shape
    tiles = torch.empty(_lib.tiles_bytes(n, k), dtype=torch.uint8, device=w.device)
    _lib.pack_tiles(w.data_ptr(), tiles.data_ptr(), n, k, stream)
    return tiles


@pytest.mark.parametrize("m,n,k,tile_n,ctas", [(16, 6144, 4096, 16, 0), (5, 2304, 8192, 16, 296), (40, 1000, 1000, 64, 37)])
def test_noalloc_matches_caller_scratch_twice(m, n, k, tile_n, ctas):
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(m * 131 + n)
    w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16).cuda()
    tiles = _packed(w, stream)
    plan = _lib.MusePlan(kernel=_lib.KERNEL_TC_STREAMK, tile_n=tile_n, ctas=ctas)
    need = _lib.scratch_bytes(m, n, k, plan)
    assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES
    scratch = torch.zeros(need, dtype=torch.uint8, device="cuda")
    for call in range(2):  # two calls in a row: the built-in area keeps the previous call's contents
        x = torch.randn((m, k), generator=g).to(torch.bfloat16).cuda()
        y_ref = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        y_na = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        _lib.proj_bf16_tiles(x.data_ptr(), tiles.data_ptr(), y_ref.data_ptr(), m, n, k, plan, stream,
                             scratch.data_ptr(), scratch.numel())
        _lib.proj_bf16_tiles_noalloc(x.data_ptr(), tiles.data_ptr(), y_na.data_ptr(), m, n, k, plan, stream)
        torch.cuda.synchronize()
        assert _lib.device_error(stream) == 0
        a, b = _bits(y_na).astype(np.uint16), _bits(y_ref).astype(np.uint16)
        rel = O.relative_l2(O.bf16_to_f32(a), O.bf16_to_f32(b))
        assert rel <= TIGHT_REL_L2, f"call {call}: relative L2 {rel:.3e} against the caller-scratch entry point"
        ok, msg, _ = O.check_implementation(_bits(x), _bits(w), a)
        assert ok, f"call {call}: {msg}"


def test_noalloc_refuses_shapes_beyond_its_area():
    m, n, k = 256, 8192, 4096
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((n, k), dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    tiles = _packed(w, stream)
    y = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    plan = _lib.MusePlan(kernel=_lib.KERNEL_TC_STREAMK, tile_n=256, ctas=148)
    assert _lib.scratch_bytes(m, n, k, plan) > _lib.NOALLOC_SCRATCH_BYTES
    with pytest.raises(_lib.MuseError) as err:
        _lib.proj_bf16_tiles_noalloc(x.data_ptr(), tiles.data_ptr(), y.data_ptr(), m, n, k, plan, stream)
    assert err.value.code == -4 and "built-in area" in str(err.value)
    with pytest.raises(_lib.MuseError) as err:  # only the stream-K kernel has a built-in scratch variant
        _lib.proj_bf16_tiles_noalloc(x.data_ptr(), tiles.data_ptr(), y.data_ptr(), m, n, k,
                                     _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE), stream)
    assert err.value.code == -7
