"""The device 12-bit encoder (muse_encode12_device + muse_encode12_device_escapes) against the host
encoder (muse_encode12), bit for bit: planes, window bases, escape offsets and entries, on ragged N,
every BF16 bit pattern, escape-dense rows and the 12-bit BASELINE config at full size; a short
escape buffer ends with device code 0x501 and no write past it; prepare(encode_on_device=True)
serves the same bits as the host-encoded path."""

import numpy as np
import pytest
import torch

from muse_bf16_proj_b200 import _lib, codec12, submission
from muse_bf16_proj_b200 import contract as C
from muse_bf16_proj_b200.dispatch import Dispatch

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _assert_same(w_bits: np.ndarray):
    enc = codec12.encode(w_bits)
    w = torch.from_numpy(w_bits.view(np.int16)).view(torch.bfloat16).cuda()
    d = submission._Enc12Device.encode_on_device(w, max_escape_fraction=1.0)
    torch.cuda.synchronize()
    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0
    assert d.n_esc == enc.n_esc
    assert np.array_equal(d.bases.cpu().numpy(), enc.bases.reshape(-1)), "window bases"
    assert np.array_equal(d.esc_ptr.cpu().numpy(), enc.esc_ptr), "escape offsets"
    assert np.array_equal(d.esc_val[: enc.n_esc].cpu().numpy().view(np.uint32), enc.esc_val), "escape entries"
    assert np.array_equal(d.planes.cpu().numpy(), enc.planes), "planes"
    return enc, d


def _normal(n, k, seed, inject=0.0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn((n, k), generator=g) * 0.02
    if inject:
        idx = torch.randperm(n * k, generator=g)[: int(n * k * inject)]
        flat = w.view(-1)
        flat[idx[: len(idx) // 2]] = 0.0
        flat[idx[len(idx) // 2:]] *= 50.0
    return _bits(w.to(torch.bfloat16))


@pytest.mark.parametrize("n,k,inject", [(1, 512, 0.0), (300, 1024, 0.001), (128, 2048, 0.01), (257, 512, 0.05),
                                        (1000, 4096, 0.001)])
def test_device_encoder_matches_host(n, k, inject):
    _assert_same(_normal(n, k, 13 * n + k, inject))


def test_device_encoder_every_bf16_pattern():
    enc, _ = _assert_same(np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(128, 512))
    assert enc.n_esc > 0


def test_device_encoder_escape_dense_rows():
    w = _normal(200, 1024, 5)
    w[17] = np.random.default_rng(3).integers(0, 65536, 1024, dtype=np.uint16)
    w[130, ::3] = 0x7F80
    _assert_same(w)


def test_device_encoder_baseline_config():
    """cfg 3's W [10240, 8192] with the BASELINE recipe (0.1 % zeros and x50 outliers)."""
    w = C.generate_baseline_weight("qkv_prefill", 1000, device="cuda", recipe="inject")
    enc, _ = _assert_same(_bits(w))
    assert 0 < enc.escape_fraction < codec12.MAX_ESCAPE_FRACTION


def test_short_escape_buffer_is_reported_not_overrun():
    n, k = 64, 512
    w_bits = _normal(n, k, 9, inject=0.05)
    enc = codec12.encode(w_bits)
    w = torch.from_numpy(w_bits.view(np.int16)).view(torch.bfloat16).cuda()
    st = torch.cuda.current_stream().cuda_stream
    planes = torch.empty(codec12.plane_bytes(n, k), dtype=torch.uint8, device="cuda")
    bases = torch.empty(k // 128, dtype=torch.uint8, device="cuda")
    esc_ptr = torch.empty(n + 1, dtype=torch.int32, device="cuda")
    _lib.encode12_device(w.data_ptr(), n, k, planes.data_ptr(), bases.data_ptr(), esc_ptr.data_ptr(), st)
    cap = enc.n_esc // 2
    assert cap > 0
    esc_val = torch.full((cap + 64,), -1, dtype=torch.int32, device="cuda")  # 64 guard words
    try:  # start from a clear error word
        _lib.device_error(st)
    except _lib.MuseError:
        pass
    _lib.encode12_device_escapes(w.data_ptr(), n, k, bases.data_ptr(), esc_ptr.data_ptr(), esc_val.data_ptr(), cap, st)
    with pytest.raises(_lib.MuseError) as err:
        _lib.device_error(st)
    assert "0x501" in str(err.value)
    got = esc_val.cpu().numpy().view(np.uint32)
    assert np.array_equal(got[:cap], enc.esc_val[:cap])
    assert (got[cap:] == 0xFFFFFFFF).all(), "an escape was written past the buffer"
    assert _lib.device_error(st) == 0


def test_prepare_encode_on_device_serves_the_same_bits():
    g = torch.Generator().manual_seed(21)
    w = (torch.randn((1024, 2048), generator=g) * 0.02).to(torch.bfloat16).cuda()
    # The smoke's table: M = 1 from the 12-bit planes, M = 2-4 and 5-256 from BF16.
    entries = [{"n": 1024, "k": 2048, "m_lo": 1, "m_hi": 1, "weights": "12b", "plan": {"kernel": "gemv_12b"}},
               {"n": 1024, "k": 2048, "m_lo": 2, "m_hi": 4, "plan": {"kernel": "gemv_bf16"}},
               {"n": 1024, "k": 2048, "m_lo": 5, "m_hi": 256, "plan": {"kernel": "tc_tile", "split": 4}}]
    host = submission.prepare({"enc": w}, dispatch=Dispatch(entries=entries), encode_12b=True, verbose=False)
    dev = submission.prepare({"enc": w}, dispatch=Dispatch(entries=entries), encode_12b=True, verbose=False,
                             encode_on_device=True)
    assert dev["enc12"]["enc"].n_esc == host["enc12"]["enc"].n_esc
    assert torch.equal(host["enc12"]["enc"].planes, dev["enc12"]["enc"].planes)
    assert torch.equal(host["enc12"]["enc"].tiles12, dev["enc12"]["enc"].tiles12)
    for m in (1, 16):
        x = torch.randn((m, 2048), generator=g).to(torch.bfloat16).cuda()
        data = {"x": x, "config": {"m": m, "n": 1024, "k": 2048, "layer": "enc"}}
        y_host = submission.kernel_fn(data, host)
        y_dev = submission.kernel_fn(data, dev)
        torch.cuda.synchronize()
        assert torch.equal(y_host, y_dev)
