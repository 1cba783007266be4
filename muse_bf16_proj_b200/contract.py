"""The problem contract on the product side: layer shapes and the seeded input generators.

This module produces the data the projections run on; it never checks results (the FP64
checker lives in the test-only ``oracle`` package). It restates the reference's generators
call for call, so the same seed gives the same tensors on the same device type:

- ``LAYERS``, ``out_features``, ``UNPOOL_SLICE`` / ``SLICED_MAX_TOKENS``: reference.py:15-24, 37-41.
- ``generate_weights``: reference.py:44-49 (std 1/sqrt(K), one generator across the layers).
- ``generate_input``: reference.py:52-69 (randn x, optional 1 %-channel x30 outliers, about one
  probe row in eight holding a single +-2^3..2^7 entry).

It adds the projection shapes the B200 build is measured on (the five configurations of the
build's baseline file) with their own recipe: W ~ N(0, 0.02) and, for the 12-bit codec case, about
0.1 % injected weight entries, half exact zeros and half x50 outliers.
"""

from __future__ import annotations

import math

import torch

# Per-GPU weights [N, K] of the reference problem (reference.py:15-21).
LAYERS = {
    "qkv_gate": (2304, 8192),
    "o": (8192, 1024),
    "pooler": (4096, 8192),
    "unpooler": (8192, 4096),
    "router": (256, 8192),
}
UNPOOL_SLICE = 1024          # reference.py:23
SLICED_MAX_TOKENS = 8        # reference.py:24
FP32_LAYERS = {"router"}     # reference.py:25
WEIGHTS_SEED = 5151          # reference.py:26
PROBE_EVERY = 8              # reference.py:33
BF16_LAYERS = tuple(name for name in LAYERS if name not in FP32_LAYERS)

# The B200 measurement shapes [N, K] (W ~ N(0, 0.02)).
BASELINE_LAYERS = {
    "qkv_decode": (6144, 4096),    # Q 4096 + K 1024 + V 1024 (GQA), decode and small-batch configs
    "qkv_prefill": (10240, 8192),  # 64 Q heads + 8 KV heads x 128, 12-bit GEMV and prefill configs
    "mlp_up": (57344, 8192),       # column-parallel MLP up/gate, sharded along N
}
BASELINE_STD = 0.02
INJECT_FRACTION = 1e-3   # of the weights: half set to exactly 0, half scaled x50
INJECT_SCALE = 50.0

# The five measured configurations: name -> (layer, M, weight recipe).
CONFIGS = {
    "decode_qkv_gemv": ("qkv_decode", 1, "normal"),
    "smallbatch_qkv": ("qkv_decode", 16, "normal"),
    "gemv12_qkv": ("qkv_prefill", 1, "inject"),
    "prefill_qkv": ("qkv_prefill", 4096, "normal"),
    "mlp_up_prefill": ("mlp_up", 8192, "normal"),
    "mlp_up_decode": ("mlp_up", 1, "normal"),
}
SMALLBATCH_SWEEP_MS = (1, 2, 4, 8, 16, 32)


def all_layers() -> dict:
    return {**LAYERS, **BASELINE_LAYERS}


def out_features(layer: str, m: int) -> int:
    """N: the output width one GPU computes for ``layer`` at ``m`` tokens (reference.py:37-41)."""
    if layer == "unpooler" and m <= SLICED_MAX_TOKENS:
        return UNPOOL_SLICE
    return all_layers()[layer][0]


def in_features(layer: str) -> int:
    return all_layers()[layer][1]


def generate_weights(seed: int = WEIGHTS_SEED, device: str = "cuda") -> dict:
    """W [N, K] for the five reference layers: N(0, 1/K), BF16 (FP32 for the router), drawn in
    LAYERS order from one generator (reference.py:44-49)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, (n, k) in LAYERS.items():
        w = torch.randn((n, k), generator=gen, device=device) / math.sqrt(k)
        out[name] = w.to(torch.float32 if name in FP32_LAYERS else torch.bfloat16)
    return out


def generate_baseline_weight(layer: str, seed: int, device: str = "cuda", recipe: str = "normal") -> torch.Tensor:
    """One measurement-shape weight, BF16 [N, K] ~ N(0, 0.02). ``recipe="inject"`` then sets a
    seeded ``INJECT_FRACTION`` of the entries (chosen by randperm) half to exactly 0 and half to
    x50 outliers. N-sharded ranks generate the whole matrix and keep their row range, so every
    world size sees the same weights."""
    n, k = BASELINE_LAYERS[layer]
    gen = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn((n, k), generator=gen, device=device) * BASELINE_STD
    if recipe == "inject":
        count = max(2, int(round(INJECT_FRACTION * n * k)))
        idx = torch.randperm(n * k, generator=gen, device=device)[:count]
        flat = w.view(-1)
        half = count // 2
        flat[idx[:half]] = 0.0
        flat[idx[half:]] *= INJECT_SCALE
    elif recipe != "normal":
        raise ValueError(f"unknown weight recipe {recipe!r}")
    return w.to(torch.bfloat16)


def generate_input(m: int, layer: str, seed: int, dist: str = "normal", device: str = "cuda", **_) -> dict:
    """x [M, K] BF16 standard normal with probe rows (reference.py:52-69): ``dist="outliers"``
    scales 1 % of the channels x30; about one row in PROBE_EVERY (and at least one at a seeded row
    when M >= PROBE_EVERY) is replaced by a single +-2^p entry, p in [3, 7]."""
    gen = torch.Generator(device=device).manual_seed(seed)
    k = in_features(layer)
    n = out_features(layer, m)
    x = torch.randn((m, k), generator=gen, device=device)
    if dist == "outliers":
        idx = torch.randperm(k, generator=gen, device=device)[: max(1, k // 100)]
        x[:, idx] *= 30
    elif dist != "normal":
        raise ValueError(f"unknown dist {dist!r}")
    probes = torch.rand((m,), generator=gen, device=device) < 1 / PROBE_EVERY
    if m >= PROBE_EVERY:
        probes[torch.randint(m, (1,), generator=gen, device=device)] = True
    cols = torch.randint(k, (m,), generator=gen, device=device)
    signs = torch.randint(2, (m,), generator=gen, device=device) * 2 - 1
    powers = torch.randint(3, 8, (m,), generator=gen, device=device)
    spike = torch.zeros_like(x).scatter_(1, cols[:, None], (signs * 2.0 ** powers).float()[:, None])
    x = torch.where(probes[:, None], spike, x)
    return {"x": x.to(torch.bfloat16), "config": {"m": m, "n": n, "k": k, "layer": layer}}
