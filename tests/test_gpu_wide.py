"""Parity of the wide-tile pair GEMM (MUSE_KERNEL_TC_WIDE: 256 tokens x 512 W rows a CTA pair,
two N = 256 UMMAs a k step into two TMEM accumulators) with the FP64 oracle.

Cases: one tile and one k block; several tiles with ragged M, N and K (token rows and W rows past
the edges are never stored; the W tiles past N are read in bounds); more tiles than CTA pairs
(persistent walk, the accumulator-0-ahead hand-over between tiles with stages kept back); every
token-tile group size (grouped order); fewer pairs than tiles; the BASELINE prefill shape on
sampled rows; determinism. Tolerances as tests/test_gpu_parity.py.
"""

import numpy as np
import pytest
import torch

from muse_bf16_proj_b200 import _lib
from oracle import contract_ref as O
from test_gpu_parity import _rand_bits, _run_bf16, assert_parity, bits, stream, to_dev

pytestmark = pytest.mark.gpu


def wide_plan(group=0, ctas=0, stages=0):
    return _lib.MusePlan(kernel=_lib.KERNEL_TC_WIDE, split=group, ctas=ctas, stages=stages)


CASES = [
    # (m, n, k, group, ctas, stages)
    (256, 512, 64, 0, 0, 0),       # one tile, one k block
    (300, 1000, 640, 0, 0, 0),     # ragged M, N, K
    (1000, 3000, 4160, 0, 0, 0),   # ragged, several tiles a pair's walk
    (2048, 4096, 2048, 2, 8, 0),   # 4 pairs walk 64 tiles: many tile hand-overs
    (2048, 4096, 2048, 1, 6, 2),   # two stages: one k block ahead at most
    (2048, 4096, 2048, 8, 0, 3),   # one group of all 8 token tiles
    (777, 2304, 8192, 0, 0, 0),    # the reference's qkv_gate at a prefill M
    (512, 57344 // 8, 1024, 0, 0, 0),  # an 8-GPU MLP shard's N
]


@pytest.mark.parametrize("m,n,k,group,ctas,stages", CASES)
def test_wide_parity(m, n, k, group, ctas, stages):
    xb, wb = _rand_bits((m, k), 11 + m + k), _rand_bits((n, k), 13 + n, 0.02)
    y = _run_bf16(xb, wb, wide_plan(group, ctas, stages), tiles=True)
    assert_parity(xb, wb, y, what=f"tc_wide m={m} n={n} k={k} group={group} ctas={ctas} stages={stages}")


def test_wide_deterministic_and_equal_to_pair_gemm():
    """Two runs bitwise equal; equal to the 256 x 256 pair GEMM on the same inputs (both sum each
    output in K order in FP32 on the tensor cores)."""
    m, n, k = 1024, 2048, 3072
    xb, wb = _rand_bits((m, k), 3), _rand_bits((n, k), 4, 0.02)
    y1 = _run_bf16(xb, wb, wide_plan(), tiles=True)
    y2 = _run_bf16(xb, wb, wide_plan(group=1, ctas=10), tiles=True)
    y3 = _run_bf16(xb, wb, _lib.MusePlan(kernel=_lib.KERNEL_TC_GEMM2), tiles=True)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert torch.equal(y1, y3)


def test_wide_prefill_config_sampled():
    """BASELINE's prefill QKV config x[4096, 8192] . W[10240, 8192]^T: 64 sampled rows against FP64,
    the whole output against a torch FP32 product (TF32 off) within BF16 rounding."""
    m, n, k = 4096, 10240, 8192
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    t = torch.empty(_lib.tiles_bytes(n, k), dtype=torch.uint8, device="cuda")
    _lib.pack_tiles(w.data_ptr(), t.data_ptr(), n, k, stream())
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    _lib.proj_bf16_tiles(x.data_ptr(), t.data_ptr(), y.data_ptr(), m, n, k, wide_plan(), stream())
    torch.cuda.synchronize()
    assert _lib.device_error(stream()) == 0
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(5))[:64]
    xs, ys = bits(x[rows]), bits(y[rows])
    ref = O.ref_kernel(xs, bits(w))
    ok, msg, _ = O.check_implementation(xs, bits(w), ys, ref_bits=ref)
    assert ok, msg
    assert O.relative_l2(O.bf16_to_f32(ys), O.bf16_to_f32(ref)) <= 1e-3
    torch.backends.cuda.matmul.allow_tf32 = False
    full = (x.float() @ w.float().t())
    rel = ((y.float() - full).norm() / full.norm()).item()
    assert rel <= 4e-3, rel
    assert np.isfinite(rel)
