"""Generates the golden fixtures in this folder by running the REFERENCE's own Python code on the CPU.

Run in a container where the reference checkout is importable (path given by --reference). The GPU
box never runs this file; the tests only read its outputs:

- contract.json: sha256 of the reference's generate_weights(5151, "cpu") per layer, and, per input
  case (layer, m, seed, dist), sha256 of generate_input(..., device="cpu")["x"] and of
  ref_kernel's BF16 output (reference.py:44-76).
- router.json: for the FP32 router, sha256 of generate_input x and of ref_kernel's FP32 output per
  case, the reference's own check verdicts, and sha256 of the BF16 hi + lo pair it builds.
- codec_ref.json: the reference's nf12_pack_cuda (submission.py:591-626) on each BF16 layer of those
  weights: c0, escape count and sha256 of every plane and escape array.
- codec_small.npz: a small W with zeros, -0, subnormals, +-inf, NaN and outliers, and the literal
  output of nf12_pack_cuda on it.
- checks_cases.npz + checks.json: outputs perturbed in seeded ways and the reference's own
  check_implementation verdicts on them (reference.py:84-99, checks.py:31-55).

Usage: python tests/golden/make_golden.py --reference <path to the reference checkout>
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (layer, m, seed, dist): the reference harness's nine tests (BF16 ones) and its scored shapes,
# with the seeds its pseudo-judge uses (7000 + m for tests, 8000 + m for scored shapes).
TEST_CASES = [("qkv_gate", 1, 7001, "normal"), ("pooler", 7, 7007, "normal"), ("o", 33, 7033, "normal"),
              ("unpooler", 130, 7130, "normal"), ("unpooler", 5, 7005, "normal"),
              ("qkv_gate", 512, 7512, "outliers"), ("unpooler", 1000, 8000, "outliers")]
SCORED_MS = (1, 8, 16, 32, 128, 256)
# The router's two harness tests (m 8 normal, m 9 outliers) and its scored shapes.
ROUTER_CASES = [(8, 7008, "normal"), (9, 7009, "outliers")] + [(m, 8000 + m, "normal") for m in SCORED_MS]
BF16_LAYERS = ("qkv_gate", "o", "pooler", "unpooler")


def sha(t) -> str:
    if isinstance(t, torch.Tensor):
        t = t.contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        t = t.numpy()
    return hashlib.sha256(np.ascontiguousarray(t).tobytes()).hexdigest()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import reference as R   # noqa: E402  (the reference's own module)
    import submission as S  # noqa: E402

    torch.manual_seed(0)
    weights = R.generate_weights(R.WEIGHTS_SEED, device="cpu")
    contract = {"weights_seed": R.WEIGHTS_SEED, "weights": {k: sha(v) for k, v in weights.items()}, "cases": []}
    cases = list(TEST_CASES) + [(layer, m, 8000 + m, "normal") for m in SCORED_MS for layer in BF16_LAYERS]
    for layer, m, seed, dist in cases:
        data = R.generate_input(m, layer, seed=seed, dist=dist, device="cpu")
        ref = R.ref_kernel(data, weights)
        ok, msg = R.check_implementation(data, ref, weights)
        contract["cases"].append({"layer": layer, "m": m, "seed": seed, "dist": dist, "n": data["config"]["n"],
                                  "k": data["config"]["k"], "x": sha(data["x"]), "ref": sha(ref),
                                  "probe_rows": int(len(R.probe_rows(data["x"]))), "self_check": [ok, msg]})
        print(layer, m, dist, msg)
    with open(os.path.join(HERE, "contract.json"), "w") as f:
        json.dump(contract, f, indent=1)

    codec = {}
    for layer in BF16_LAYERS:
        p = S.nf12_pack_cuda(weights[layer])
        codec[layer] = {"c0": p["c0"], "escapes": p["escapes"], "lo": sha(p["lo"]), "nib": sha(p["nib"]),
                        "esc_ptr": sha(p["esc_ptr"]), "esc_k": sha(p["esc_k"]), "esc_delta": sha(p["esc_delta"])}
        print("nf12", layer, p["c0"], p["escapes"])
    with open(os.path.join(HERE, "codec_ref.json"), "w") as f:
        json.dump(codec, f, indent=1)

    # The FP32 router: its two harness tests and scored shapes (FP32 output), and the BF16 hi + lo
    # pair the reference builds in prepare (submission.py:1120-1124).
    router = {"cases": []}
    for m, seed, dist in ROUTER_CASES:
        data = R.generate_input(m, "router", seed=seed, dist=dist, device="cpu")
        ref = R.ref_kernel(data, weights)
        ok, msg = R.check_implementation(data, ref, weights)
        router["cases"].append({"m": m, "seed": seed, "dist": dist, "n": data["config"]["n"], "k": data["config"]["k"],
                                "x": sha(data["x"]), "ref": sha(ref), "ref_dtype": str(ref.dtype),
                                "probe_rows": int(len(R.probe_rows(data["x"]))), "self_check": [ok, msg]})
        print("router", m, dist, msg)
    hi = weights["router"].to(torch.bfloat16)
    lo = (weights["router"] - hi.float()).to(torch.bfloat16)
    router["hi"], router["lo"] = sha(hi), sha(lo)
    with open(os.path.join(HERE, "router.json"), "w") as f:
        json.dump(router, f, indent=1)

    # A small W with special values, packed by the reference.
    gen = torch.Generator(device="cpu").manual_seed(1234)
    w = (torch.randn((32, 1024), generator=gen) * 0.02)
    flat = w.view(-1)
    idx = torch.randperm(w.numel(), generator=gen)[:48]
    specials = [0.0, -0.0, 1e-40, -1e-40, float("inf"), float("-inf"), 3.0, -7.5, 1e-30, 2.0 ** -20, 65504.0, 1e20]
    for j, i in enumerate(idx.tolist()):
        flat[i] = specials[j % len(specials)]
    w = w.to(torch.bfloat16)
    p = S.nf12_pack_cuda(w)
    np.savez_compressed(os.path.join(HERE, "codec_small.npz"), w=bits(w), lo=p["lo"].numpy(), nib=p["nib"].numpy(),
                        c0=np.int32(p["c0"]), esc_ptr=p["esc_ptr"].numpy(), esc_k=p["esc_k"].numpy(),
                        esc_delta=p["esc_delta"].numpy())
    print("small codec", p["c0"], p["escapes"])

    # check_implementation on seeded perturbations of a small synthetic layer.
    gen = torch.Generator(device="cpu").manual_seed(99)
    wt = (torch.randn((128, 512), generator=gen) / 32).to(torch.bfloat16)
    fake = {"fakelayer": wt}
    x = torch.randn((64, 512), generator=gen)
    x[3] = 0
    x[3, 77] = 16.0   # a probe row
    x = x.to(torch.bfloat16)
    data = {"x": x, "config": {"m": 64, "n": 128, "k": 512, "layer": "fakelayer"}}
    ref = R.ref_kernel(data, fake)
    outs = {}
    outs["exact"] = ref.clone()
    outs["noise_small"] = (ref.float() * (1 + 1e-3 * torch.randn(ref.shape, generator=gen))).to(torch.bfloat16)
    outs["noise_big"] = (ref.float() * (1 + 3e-2 * torch.randn(ref.shape, generator=gen))).to(torch.bfloat16)
    bad_row = ref.float().clone()
    bad_row[5] *= 1.07  # the whole output passes, this row does not
    outs["bad_row"] = bad_row.to(torch.bfloat16)
    probe_off = ref.float().clone()
    probe_off[3] *= 1.004
    outs["probe_off"] = probe_off.to(torch.bfloat16)
    nan = ref.float().clone()
    nan[0, 0] = float("nan")
    outs["nan"] = nan.to(torch.bfloat16)
    verdicts = {}
    for name, out in outs.items():
        ok, msg = R.check_implementation(data, out, fake)
        verdicts[name] = [ok, msg]
        print("check", name, ok, msg)
    np.savez_compressed(os.path.join(HERE, "checks_cases.npz"), w=bits(wt), x=bits(x), ref=bits(ref),
                        **{f"out_{k}": bits(v) for k, v in outs.items()})
    with open(os.path.join(HERE, "checks.json"), "w") as f:
        json.dump(verdicts, f, indent=1)


if __name__ == "__main__":
    main()
