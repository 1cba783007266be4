"""The five measured configurations at full size, on one GPU.

Small outputs are checked in full against the FP64 oracle. The prefill-sized outputs are checked
(1) on a seeded sample of output rows x weight rows against the FP64 oracle, with the reference's
check and the tighter relative-L2 bound of test_gpu_parity, and (2) in full against a torch FP32
product on the GPU (TF32 off) within relative L2 1e-3 (both round to BF16 last).
"""

import numpy as np
import pytest
import torch

from muse_bf16_proj_b200 import _lib, submission
from muse_bf16_proj_b200 import contract as C
from muse_bf16_proj_b200.dispatch import Dispatch
from oracle import contract_ref as O

from test_gpu_parity import assert_parity, bits

pytestmark = pytest.mark.gpu


def _state(layer, recipe="normal", seed=1, entries=None, encode_12b=None):
    w = C.generate_baseline_weight(layer, seed, device="cuda", recipe=recipe)
    disp = Dispatch(entries=entries) if entries is not None else Dispatch()
    return w, submission.prepare({layer: w}, dispatch=disp, encode_12b=encode_12b, verbose=False)


def _sampled_check(x, w, y, rows=64, cols=1024, seed=0):
    g = torch.Generator().manual_seed(seed)
    ri = torch.randperm(x.shape[0], generator=g)[:rows].sort().values
    ci = torch.randperm(w.shape[0], generator=g)[:cols].sort().values
    xs, ws = bits(x[ri.cuda()]), bits(w[ci.cuda()])
    ys = y[ri.cuda()][:, ci.cuda()]
    assert_parity(xs, ws, ys, what="sampled")


def _fp32_check(x, w, y, tol=1e-3):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = (x.float() @ w.float().T).to(torch.bfloat16).float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    rel = ((y.float() - ref).norm() / ref.norm()).item()
    assert torch.isfinite(y.float()).all()
    assert rel <= tol, f"relative L2 vs FP32 {rel:.3e}"


@pytest.mark.parametrize("m", C.SMALLBATCH_SWEEP_MS)
def test_decode_and_smallbatch_qkv(m):
    w, st = _state("qkv_decode")
    data = C.generate_input(m, "qkv_decode", 100 + m, device="cpu")
    y = submission.kernel_fn({"x": data["x"].cuda(), "config": data["config"]}, st)
    assert_parity(bits(data["x"]), bits(w), y, what=f"qkv_decode m={m}")


def test_gemv12_qkv_prefill_inject():
    entries = [{"n": 10240, "k": 8192, "m_lo": 1, "m_hi": 1, "weights": "12b", "plan": {"kernel": "gemv_12b"}}]
    w, st = _state("qkv_prefill", recipe="inject", seed=3, entries=entries)
    enc = st["enc12"]["qkv_prefill"]
    assert 0.0008 < enc.escape_fraction < 0.0015
    data = C.generate_input(1, "qkv_prefill", 301, device="cpu")
    y = submission.kernel_fn({"x": data["x"].cuda(), "config": data["config"]}, st)
    assert_parity(bits(data["x"]), bits(w), y, what="gemv12 qkv_prefill")
    # the same weights through the BF16 path agree to within output rounding
    y16 = torch.empty_like(y)
    _lib.proj_bf16(data["x"].cuda().data_ptr(), w.data_ptr(), y16.data_ptr(), 1, 10240, 8192,
                   _lib.MusePlan(kernel=_lib.KERNEL_GEMV_BF16), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert O.relative_l2(y.float().cpu().numpy(), y16.float().cpu().numpy()) < 1e-3


def test_prefill_qkv_full():
    w, st = _state("qkv_prefill", seed=4)
    data = C.generate_input(4096, "qkv_prefill", 401, device="cuda")
    x = data["x"]
    y = submission.kernel_fn(data, st)
    torch.cuda.synchronize()
    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0
    _sampled_check(x, w, y)
    _fp32_check(x, w, y)


@pytest.mark.parametrize("m", [1, 8192])
def test_mlp_up_single_gpu(m):
    w, st = _state("mlp_up", seed=5)
    data = C.generate_input(m, "mlp_up", 500 + m, device="cuda")
    x = data["x"]
    y = submission.kernel_fn(data, st)
    torch.cuda.synchronize()
    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0
    if m == 1:
        assert_parity(bits(x), bits(w), y, what="mlp_up m=1")
    else:
        _sampled_check(x, w, y)
        _fp32_check(x, w, y)
