"""Pins the CPU oracle (and the product-side generators) to fixtures made by the reference itself.

tests/golden/make_golden.py ran the reference's reference.py / submission.py on the CPU; these
tests recompute everything with this repo's code and compare bit for bit.
"""

import hashlib
import json
import os

import numpy as np
import pytest
import torch

from muse_bf16_proj_b200 import contract as C
from oracle import codec12_ref as Q
from oracle import contract_ref as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLD, "contract.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def weights():
    return C.generate_weights(C.WEIGHTS_SEED, device="cpu")


def test_weights_match_reference(golden, weights):
    for name, w in weights.items():
        b = bits(w) if w.dtype == torch.bfloat16 else w.numpy()
        assert sha(b) == golden["weights"][name], name


def test_inputs_and_fp64_outputs_match_reference(golden, weights):
    checked = 0
    for case in golden["cases"]:
        data = C.generate_input(case["m"], case["layer"], case["seed"], case["dist"], device="cpu")
        xb = bits(data["x"])
        assert sha(xb) == case["x"], case
        assert data["config"]["n"] == case["n"] and data["config"]["k"] == case["k"]
        assert len(O.probe_rows(xb)) == case["probe_rows"]
        if case["m"] <= 256:  # the FP64 product of the two largest cases takes minutes here
            ref = O.ref_kernel(xb, bits(weights[case["layer"]]), case["n"])
            assert sha(ref) == case["ref"], case
            checked += 1
    assert checked >= 25


def test_router_inputs_fp32_outputs_and_hi_lo_match_reference(weights):
    """The FP32 router: generate_input x, the FP64-then-FP32 reference output, the reference's
    own check verdicts on it, and the BF16 hi + lo pair of its prepare step."""
    with open(os.path.join(GOLD, "router.json")) as f:
        gold = json.load(f)
    w = weights["router"].numpy()
    assert w.dtype == np.float32 and w.shape == (256, 8192)
    for case in gold["cases"]:
        data = C.generate_input(case["m"], "router", case["seed"], case["dist"], device="cpu")
        xb = bits(data["x"])
        assert sha(xb) == case["x"], case
        assert len(O.probe_rows(xb)) == case["probe_rows"]
        ref = O.ref_kernel_f32(xb, w, case["n"])
        assert ref.dtype == np.float32 and sha(ref) == case["ref"], case
        ok, _, _ = O.check_implementation_f32(xb, w, ref, case["n"])
        assert ok == case["self_check"][0]
    hi, lo = O.split_hi_lo(w)
    assert sha(hi) == gold["hi"] and sha(lo) == gold["lo"]


def test_router_check_rejects_bf16_weights(weights):
    """The reference's reason for hi + lo: BF16 router weights alone fail the 1e-4 tolerance,
    hi + lo with FP32 accumulation passes."""
    w = weights["router"].numpy()
    data = C.generate_input(16, "router", 8016, "normal", device="cpu")
    xb = bits(data["x"])
    x = O.bf16_to_f32(xb).astype(np.float64)
    hi, lo = O.split_hi_lo(w)
    out_bf16 = (x @ O.bf16_to_f32(hi).astype(np.float64).T).astype(np.float32)
    out_hilo = (x @ (O.bf16_to_f32(hi).astype(np.float64) + O.bf16_to_f32(lo).astype(np.float64)).T).astype(np.float32)
    assert not O.check_implementation_f32(xb, w, out_bf16)[0]
    assert O.check_implementation_f32(xb, w, out_hilo)[0]


def test_reference_codec_matches_nf12_pack(weights):
    with open(os.path.join(GOLD, "codec_ref.json")) as f:
        g = json.load(f)
    for layer, e in g.items():
        p = Q.pack_reference(bits(weights[layer]))
        assert p["c0"] == e["c0"] and p["escapes"] == e["escapes"], layer
        for key in ("lo", "nib", "esc_ptr", "esc_k", "esc_delta"):
            assert sha(p[key]) == e[key], (layer, key)


def test_reference_codec_small_special_values():
    d = np.load(os.path.join(GOLD, "codec_small.npz"))
    p = Q.pack_reference(d["w"])
    assert p["c0"] == int(d["c0"])
    for key in ("lo", "nib", "esc_ptr", "esc_k"):
        assert np.array_equal(p[key], d[key]), key
    assert np.array_equal(p["esc_delta"].view(np.uint32), d["esc_delta"].view(np.uint32))
    # The reference format rebuilds every in-window weight bit for bit. Its escapes carry an FP32
    # delta from the placeholder, which loses -0, subnormals and values far below the placeholder
    # (they come back as +0): those escapes are exact only in value up to the placeholder's
    # rounding. The build's own format stores escaped weights' bits (test_codec12 checks all 65,536).
    back = Q.unpack_reference(p)
    w = d["w"]
    esc = np.zeros(w.shape, dtype=bool)
    rows = np.repeat(np.arange(w.shape[0]), np.diff(p["esc_ptr"]))
    esc[rows, p["esc_k"]] = True
    assert np.array_equal(back[~esc], w[~esc])
    lossy = int(np.count_nonzero(back[esc] != w[esc]))
    assert 0 < lossy < esc.sum()
    f = lambda b: (b.astype(np.uint32) << 16).view(np.float32)
    placeholder = f(np.array([int(d["c0"]) << 8], dtype=np.uint16))[0]
    finite = np.isfinite(f(w[esc]))
    assert np.all(np.abs(f(back[esc])[finite] - f(w[esc])[finite]) <= np.abs(placeholder) * 2.0 ** -23
                  + np.abs(f(w[esc])[finite]) * 2.0 ** -8)


def test_tile_format_with_one_tile_equals_reference_planes():
    """With a single window for the whole matrix the per-tile format holds the reference's bytes."""
    d = np.load(os.path.join(GOLD, "codec_small.npz"))
    w = d["w"]
    enc = Q.encode_tiles(w, tile_r=w.shape[0], tile_k=w.shape[1])
    assert int(enc["bases"][0, 0]) == int(d["c0"])
    assert np.array_equal(enc["lo"], d["lo"])
    code = enc["code"].astype(np.int32)
    assert np.array_equal((code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8), d["nib"])
    rows = np.repeat(np.arange(w.shape[0]), np.diff(enc["esc_ptr"]))
    assert np.array_equal(enc["esc_ptr"], d["esc_ptr"])
    assert np.array_equal((enc["esc_val"] >> 16).astype(np.int32), d["esc_k"])
    assert len(rows) == len(d["esc_k"])


def test_check_implementation_matches_reference_verdicts():
    d = np.load(os.path.join(GOLD, "checks_cases.npz"))
    with open(os.path.join(GOLD, "checks.json")) as f:
        verdicts = json.load(f)
    ref = O.ref_kernel(d["x"], d["w"])
    assert np.array_equal(ref, d["ref"])
    for name, (ok_ref, msg_ref) in verdicts.items():
        ok, msg, _ = O.check_implementation(d["x"], d["w"], d["out_" + name], ref_bits=ref)
        assert ok == ok_ref, (name, msg, msg_ref)
