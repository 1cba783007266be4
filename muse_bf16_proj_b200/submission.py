"""The drop-in entry point for the dense projections: ``prepare(weights)`` once, untimed, then
``kernel_fn(data, state)`` per call (the reference's interface, submission.py:23-41, 1115-1173).

What serves each shape (``kernel_fn`` -> ``project``), chosen per (N, K, M) by the committed sweep
table (``dispatch.py``), else by the library's default plan (muse_plan_default):

- BF16 W, few tokens: the tcgen05 tile kernel on packed W tiles with K split across CTAs (partials
  reduced in rank order by the last CTA), stream-K variants (W as the UMMA's A or B operand) for
  large N, and a streaming CUDA-core GEMV where it wins;
- BF16 W, prefill: persistent tcgen05 GEMMs (CTA pairs with cta_group::2 past M = 256);
- 12-bit W (opt-in or table rows): lossless 12-bit blocks decoded to BF16 in shared memory and fed
  to the tensor cores, or the CUDA-core 12-bit GEMV;
- the FP32 router: W in FP32 on CUDA cores up to 4 tokens, else its BF16 hi + lo pair as one
  K = 2K tensor-core projection with FP32 accumulation and output (submission.py:1027-1076).

All are this build's own sm_100a kernels behind the C ABI in include/muse_proj.h. There is no
cuBLAS, Triton or CPU fallback: a shape the kernels cannot run raises.

``prepare`` keeps every weight resident, packs the tile copies the tensor-core kernels stream
(the router's as hi | lo), builds 12-bit copies of the layers the table serves from 12 bits (host
encoder, checked lossless bit for bit), and runs a known-answer self-check of every planned kernel:
one-hot power-of-two rows of x must return exact columns of W (the reference's probe-row idea,
reference.py:30-35; within 1e-5 for the router's hi + lo), so a wrong kernel raises in prepare
instead of serving (the reference instead fell back to Triton/cuBLAS, submission.py:1142-1151).
"""

from __future__ import annotations

import os
from typing import TypedDict

import numpy as np
import torch

from . import _lib, codec12
from .contract import UNPOOL_SLICE, SLICED_MAX_TOKENS
from .dispatch import Dispatch


# Split-K scratch allocated in prepare (counters + FP32 partials); grown on demand outside capture.
SCRATCH_BYTES = 8 * 1024 * 1024


class Weights(TypedDict):
    qkv_gate: torch.Tensor  # bfloat16 [2304, 8192]
    o: torch.Tensor         # bfloat16 [8192, 1024]
    pooler: torch.Tensor    # bfloat16 [4096, 8192]
    unpooler: torch.Tensor  # bfloat16 [8192, 4096]; up to 8 tokens, only rows 0-1023 (this GPU's slice)
    router: torch.Tensor    # float32 [256, 8192]; FP32 output


class Config(TypedDict):
    m: int
    n: int      # output width; the unpooler's is 1024 up to 8 tokens (this GPU's slice), else 8192
    k: int
    layer: str  # which weight


class Inputs(TypedDict):
    x: torch.Tensor  # bfloat16 [M, K] (the router's too: its weights and output are FP32)
    config: Config


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


class _Enc12Device:
    """A 12-bit encoded weight resident on the device, with C-ABI views per output width n."""

    def __init__(self, enc: codec12.Encoded12, device: torch.device):
        self.n, self.k, self.n_esc = enc.n, enc.k, enc.n_esc
        self.planes = torch.from_numpy(enc.planes).to(device)
        self.bases = torch.from_numpy(enc.bases.reshape(-1)).to(device)
        self.esc_ptr = torch.from_numpy(enc.esc_ptr).to(device)
        self.esc_val = torch.from_numpy(enc.esc_val.view(np.int32) if enc.n_esc else np.zeros(1, np.int32)).to(device)
        self.escape_fraction = enc.escape_fraction
        self._esc_ptr_host = enc.esc_ptr
        self._views: dict = {}
        # The same weights re-laid in 12 KB blocks of 128 rows x 64 k for the tensor-core kernel.
        self.tiles12 = torch.empty(_lib.tiles12_bytes(enc.n, enc.k), dtype=torch.uint8, device=device)
        _lib.pack_tiles12(self.view(enc.n), self.tiles12.data_ptr(), torch.cuda.current_stream(device).cuda_stream)

    @classmethod
    def encode_on_device(cls, w: torch.Tensor, max_escape_fraction: float = codec12.MAX_ESCAPE_FRACTION):
        """Encodes BF16 W [N, K] on its GPU (muse_encode12_device: the host encoder's format and bits,
        without W's trip through host memory). None when more than `max_escape_fraction` of the
        weights escape (the escapes are then not written)."""
        n, k = w.shape
        dev = w.device
        st = torch.cuda.current_stream(dev).cuda_stream
        planes = torch.empty(codec12.plane_bytes(n, k), dtype=torch.uint8, device=dev)
        bases = torch.empty(-(-n // codec12.TILE) * (k // codec12.TILE), dtype=torch.uint8, device=dev)
        esc_ptr = torch.empty(n + 1, dtype=torch.int32, device=dev)
        _lib.encode12_device(w.data_ptr(), n, k, planes.data_ptr(), bases.data_ptr(), esc_ptr.data_ptr(), st)
        esc_ptr_host = esc_ptr.cpu().numpy()  # waits for step 1: the escape count sizes step 2
        n_esc = int(esc_ptr_host[n])
        if n_esc > max_escape_fraction * n * k:
            return None
        esc_val = torch.zeros(max(n_esc, 1), dtype=torch.int32, device=dev)
        if n_esc:
            _lib.encode12_device_escapes(w.data_ptr(), n, k, bases.data_ptr(), esc_ptr.data_ptr(), esc_val.data_ptr(),
                                         n_esc, st)
        _lib.device_error(st)  # raises if an escape fell outside its range
        self = cls.__new__(cls)
        self.n, self.k, self.n_esc = n, k, n_esc
        self.planes, self.bases, self.esc_ptr, self.esc_val = planes, bases, esc_ptr, esc_val
        self.escape_fraction = n_esc / float(n * k)
        self._esc_ptr_host = esc_ptr_host
        self._views = {}
        self.tiles12 = torch.empty(_lib.tiles12_bytes(n, k), dtype=torch.uint8, device=dev)
        _lib.pack_tiles12(self.view(n), self.tiles12.data_ptr(), st)
        return self

    def to_host(self) -> codec12.Encoded12:
        """The encoding as host arrays (for the on-disk cache)."""
        bases = self.bases.cpu().numpy().reshape(-(-self.n // codec12.TILE), self.k // codec12.TILE)
        esc_val = self.esc_val[:self.n_esc].cpu().numpy().view(np.uint32).copy()
        return codec12.Encoded12(self.planes.cpu().numpy(), bases, self._esc_ptr_host.copy(), esc_val, self.n, self.k)

    def view(self, n: int) -> _lib.MuseEnc12:
        v = self._views.get(n)
        if v is None:
            v = _lib.MuseEnc12(self.planes.data_ptr(), self.bases.data_ptr(), self.esc_ptr.data_ptr(),
                               self.esc_val.data_ptr(), n, self.k, int(self._esc_ptr_host[n]))
            self._views[n] = v
        return v

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.planes, self.tiles12, self.bases, self.esc_ptr,
                                                          self.esc_val))


def _encode12_on_device(w: torch.Tensor, cache_dir: str | None):
    """(_Enc12Device or None when too many weights escape, from_cache) for BF16 W on the GPU:
    from cache_dir's file for this exact weight when there is one, else encoded on the device (and
    written there for the next process)."""
    path = key = None
    if cache_dir:
        key = codec12.weight_key(_bits(w))
        path = os.path.join(cache_dir, f"{key}.m12")
        enc = codec12.load(path, key)
        if enc is not None and (enc.n, enc.k) == tuple(w.shape):
            return _Enc12Device(enc, w.device), True
    dev_enc = _Enc12Device.encode_on_device(w)
    if dev_enc is not None and path is not None:
        os.makedirs(cache_dir, exist_ok=True)
        codec12.save(dev_enc.to_host(), path, key)
    return dev_enc, False


def prepare(weights: dict, dispatch: Dispatch | None = None, encode_12b: bool | None = None,
            self_check: bool = True, verbose: bool = True, pdl: bool = True, cache_dir: str | None = None,
            encode_on_device: bool = False) -> dict:
    """Builds the state kernel_fn serves from. ``weights``: name -> W [N, K] on the GPU (BF16, or
    FP32 for the router). ``encode_12b`` forces (True) or forbids (False) the 12-bit copies; None
    lets the dispatch table decide. ``cache_dir`` (or $MUSE_12B_CACHE): where 12-bit encodings are
    kept between processes (one file per weight, keyed by the weight's hash; a stale or foreign
    file is ignored and rewritten). ``encode_on_device``: encode on the GPU (muse_encode12_device,
    the same bits) instead of the host encoder with its decode round trip; the known-answer
    self-check still runs on every planned kernel."""
    _lib.load()
    disp = dispatch if dispatch is not None else Dispatch()
    state = {"weights": {}, "tiles": {}, "fp32": {}, "fp32_tiles": {}, "enc12": {}, "dispatch": disp, "checked": [],
             "scratch": None, "scratch_need": {}, "pdl": pdl, "pdl_plans": {}}
    for name, w in weights.items():
        if w.dtype == torch.float32:
            if w.dim() != 2 or not w.is_cuda:
                raise ValueError(f"{name}: expected a 2-D CUDA tensor, got {tuple(w.shape)} on {w.device}")
            w = w.contiguous()
            state["fp32"][name] = w
            n, k = w.shape
            # The BF16 hi + lo pair (hi = BF16(W), lo = BF16(W - hi)) as the tiles of [hi | lo].
            tiles = torch.empty(_lib.router_tiles_bytes(n, k), dtype=torch.uint8, device=w.device)
            _lib.pack_router(w.data_ptr(), tiles.data_ptr(), n, k, torch.cuda.current_stream(w.device).cuda_stream)
            state["fp32_tiles"][name] = tiles
            continue
        if w.dtype != torch.bfloat16:
            raise ValueError(f"{name}: weights must be bfloat16 or float32, got {w.dtype}")
        if w.dim() != 2 or not w.is_cuda:
            raise ValueError(f"{name}: expected a 2-D CUDA tensor, got {tuple(w.shape)} on {w.device}")
        w = w.contiguous()
        state["weights"][name] = w
        n, k = w.shape
        if k % 8 == 0:  # the tensor-core path streams W from contiguous swizzled 16 KB tiles
            tiles = torch.empty(_lib.tiles_bytes(n, k), dtype=torch.uint8, device=w.device)
            _lib.pack_tiles(w.data_ptr(), tiles.data_ptr(), n, k, torch.cuda.current_stream(w.device).cuda_stream)
            state["tiles"][name] = tiles
        widths = [n] + ([UNPOOL_SLICE] if name == "unpooler" and n > UNPOOL_SLICE else [])
        want = encode_12b if encode_12b is not None else any(disp.wants_12b(nn, k) for nn in widths)
        if want and k % codec12.UNIT == 0 and k <= 65536:
            if encode_on_device:
                dev_enc, cached = _encode12_on_device(w, cache_dir or os.environ.get("MUSE_12B_CACHE"))
                if dev_enc is None or dev_enc.escape_fraction > codec12.MAX_ESCAPE_FRACTION:
                    if verbose:
                        print(f"muse: {name}: over {codec12.MAX_ESCAPE_FRACTION:.0%} escapes, kept BF16 only")
                else:
                    state["enc12"][name] = dev_enc
                    if verbose:
                        print(f"muse: {name}: 12-bit planes ({'cached' if cached else 'encoded on the device'}), "
                              f"{dev_enc.n_esc} escapes ({dev_enc.escape_fraction:.4%})")
                continue
            # From cache_dir's file for this exact weight when there is one, else encoded (raises if
            # the round trip is not bit-exact) and written there for the next process.
            enc, cached = codec12.encode_cached(_bits(w), cache_dir or os.environ.get("MUSE_12B_CACHE"))
            if enc.escape_fraction > codec12.MAX_ESCAPE_FRACTION:
                if verbose:
                    print(f"muse: {name}: {enc.escape_fraction:.3%} escapes, kept BF16 only")
            else:
                state["enc12"][name] = _Enc12Device(enc, w.device)
                if verbose:
                    print(f"muse: {name}: 12-bit planes{' (cached)' if cached else ''}, {enc.n_esc} escapes "
                          f"({enc.escape_fraction:.4%})")
    state["scratch"] = torch.zeros(SCRATCH_BYTES, dtype=torch.uint8, device=next(iter(state["weights"].values())).device
                                   if state["weights"] else "cuda")
    if self_check:
        for name, w in state["weights"].items():
            n, k = w.shape
            for nn, ms in _check_points(name, n, k, disp):
                for m in ms:
                    _known_answer_check(state, name, nn, m)
                    state["checked"].append((name, nn, m))
        for name, w in state["fp32"].items():
            for m in (1, 4, 5, 16):  # both FP32 plans: CUDA cores up to 4 tokens, hi + lo above
                _known_answer_check_f32(state, name, m)
                state["checked"].append((name, w.shape[0], m))
    torch.cuda.synchronize()
    return state


def _check_points(name: str, n: int, k: int, disp: Dispatch):
    """(n, [m, ...]) pairs the self-check runs: each table row's range ends, plus 1 and 16."""
    widths = [n] + ([UNPOOL_SLICE] if name == "unpooler" and n > UNPOOL_SLICE else [])
    out = []
    for nn in widths:
        ms = {1, 16} if nn == n else {1, SLICED_MAX_TOKENS}
        for lo, hi, _ in disp.ms_for(nn, k):
            ms.update({lo, min(hi, 256)})
        if nn == UNPOOL_SLICE and name == "unpooler":
            ms = {m for m in ms if m <= SLICED_MAX_TOKENS}
        out.append((nn, sorted(ms)))
    return out


def _known_answer_check(state: dict, layer: str, n: int, m: int) -> None:
    """x = one-hot rows (value 2^p at a spread column): y row i must be 2^p * W[:n, c_i]."""
    w = state["weights"][layer]
    k = w.shape[1]
    dev = w.device
    cols = (torch.arange(m, device=dev) * 7919 + 17) % k
    powers = 2.0 ** (torch.arange(m, device=dev) % 5)
    x = torch.zeros((m, k), dtype=torch.float32, device=dev)
    x[torch.arange(m, device=dev), cols] = powers
    x = x.to(torch.bfloat16)
    y = project(x, state, layer, n).float()
    expect = (w[:n].float()[:, cols].T * powers[:, None]).to(torch.bfloat16).float()
    plan, fmt = state["dispatch"].plan(m, n, k, layer in state["enc12"], tiles=layer in state["tiles"])
    if fmt == "12b":
        err = ((y - expect).norm(dim=1) / expect.norm(dim=1).clamp(min=1e-30)).max().item()
        ok = err <= 1e-3
    else:
        ok = torch.equal(y, expect) or bool(((y == expect) | (torch.isnan(y) & torch.isnan(expect))).all())
        err = (y - expect).abs().max().item()
    code = _lib.device_error(torch.cuda.current_stream(dev).cuda_stream)
    if not ok or code:
        raise RuntimeError(f"muse self-check failed: {layer} n={n} m={m} plan={plan.as_dict()} {fmt}: "
                           f"err {err:.3e}, device error {code:#x}")


def _known_answer_check_f32(state: dict, layer: str, m: int) -> None:
    """The router's one-hot check: row i of y must be 2^p * W[:, c_i] (exact on the FP32 kernel,
    within 1e-5 relative on hi + lo, whose rounding is ~2^-17 of each weight)."""
    w = state["fp32"][layer]
    n, k = w.shape
    dev = w.device
    cols = (torch.arange(m, device=dev) * 7919 + 17) % k
    powers = 2.0 ** (torch.arange(m, device=dev) % 5)
    x = torch.zeros((m, k), dtype=torch.float32, device=dev)
    x[torch.arange(m, device=dev), cols] = powers
    y = project_f32(x.to(torch.bfloat16), state, layer)
    expect = w[:, cols].T * powers[:, None]
    plan = _plan_f32(state, m, n, k)
    if plan.kernel == _lib.KERNEL_F32_GEMV:
        ok, err = torch.equal(y, expect), (y - expect).abs().max().item()
    else:
        err = ((y - expect).norm(dim=1) / expect.norm(dim=1).clamp(min=1e-30)).max().item()
        ok = err <= 1e-5
    code = _lib.device_error(torch.cuda.current_stream(dev).cuda_stream)
    if not ok or code:
        raise RuntimeError(f"muse self-check failed: {layer} m={m} plan={plan.as_dict()}: err {err:.3e}, "
                           f"device error {code:#x}")


def _plan_f32(state: dict, m: int, n: int, k: int) -> _lib.MusePlan:
    key = ("f32", m, n, k)
    plan = state["pdl_plans"].get(key)
    if plan is None:
        plan = _lib.plan_default(m, n, k, f32=True)
        if state.get("pdl", True):
            plan = _lib.MusePlan.from_dict({**plan.as_dict(), "flags": plan.flags | _lib.FLAG_PDL})
        state["pdl_plans"][key] = plan
    return plan


def project_f32(x: torch.Tensor, state: dict, layer: str, n: int | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ W[:n].T for an FP32 W (the router): FP32 [m, n]."""
    w = state["fp32"][layer]
    big_n, k = w.shape
    n = big_n if n is None else n
    if x.dim() != 2 or x.shape[1] != k or x.dtype != torch.bfloat16 or not (0 < n <= big_n):
        raise ValueError(f"{layer}: x {tuple(x.shape)} {x.dtype}, n={n} does not match W {tuple(w.shape)}")
    if x.device != w.device:
        raise ValueError(f"{layer}: x is on {x.device}, W on {w.device}")
    if not x.is_contiguous():
        x = x.contiguous()
    if x.data_ptr() % 16:
        x = x.clone()
    m = x.shape[0]
    plan = _plan_f32(state, m, n, k)
    y = out if out is not None else torch.empty((m, n), dtype=torch.float32, device=x.device)
    scratch = _scratch_for(state, m, n, k, plan)
    _lib.proj_f32(x.data_ptr(), w.data_ptr(), state["fp32_tiles"][layer].data_ptr(), y.data_ptr(), m, n, k, plan,
                  torch.cuda.current_stream(x.device).cuda_stream, scratch.data_ptr() if scratch is not None else 0,
                  scratch.numel() if scratch is not None else 0)
    return y


def project(x: torch.Tensor, state: dict, layer: str, n: int | None = None,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ W[:n].T on this build's kernels: BF16 [m, n], FP32 for an FP32 W (the router)."""
    if layer in state["fp32"]:
        return project_f32(x, state, layer, n, out)
    w = state["weights"].get(layer)
    if w is None:
        raise KeyError(layer)
    big_n, k = w.shape
    n = big_n if n is None else n
    if x.dim() != 2 or x.shape[1] != k or x.dtype != torch.bfloat16 or not (0 < n <= big_n):
        raise ValueError(f"{layer}: x {tuple(x.shape)} {x.dtype}, n={n} does not match W {tuple(w.shape)}")
    if x.device != w.device:
        raise ValueError(f"{layer}: x is on {x.device}, W on {w.device}")
    if not x.is_contiguous():
        x = x.contiguous()
    if x.data_ptr() % 16:
        x = x.clone()  # the kernels read x with 16-byte vector loads / TMA
    m = x.shape[0]
    enc = state["enc12"].get(layer)
    plan, fmt = state["dispatch"].plan(m, n, k, enc is not None, tiles=layer in state["tiles"])
    if state.get("pdl", True) and not plan.flags & _lib.FLAG_PDL:
        # The weights are prepare-time constants, so the kernel may stream them before the
        # previous kernel in the stream has finished (programmatic dependent launch).
        plan = state["pdl_plans"].setdefault(plan.key(), _lib.MusePlan.from_dict({**plan.as_dict(),
                                                                                "flags": plan.flags | _lib.FLAG_PDL}))
    y = out if out is not None else torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    if fmt == "12b" and plan.kernel in (_lib.KERNEL_TC_12B, _lib.KERNEL_GEMV_12T):
        scratch = _scratch_for(state, m, n, k, plan)
        _lib.proj_12b_tiles(enc.view(n), enc.tiles12.data_ptr(), x.data_ptr(), y.data_ptr(), m, plan, stream,
                            scratch.data_ptr() if scratch is not None else 0,
                            scratch.numel() if scratch is not None else 0)
    elif fmt == "12b":
        _lib.proj_12b(enc.view(n), x.data_ptr(), y.data_ptr(), m, plan, stream)
    elif plan.kernel in _lib.TILE_KERNELS and layer in state["tiles"]:
        scratch = _scratch_for(state, m, n, k, plan)
        _lib.proj_bf16_tiles(x.data_ptr(), state["tiles"][layer].data_ptr(), y.data_ptr(), m, n, k, plan, stream,
                             scratch.data_ptr() if scratch is not None else 0,
                             scratch.numel() if scratch is not None else 0)
    else:
        scratch = _scratch_for(state, m, n, k, plan)
        _lib.proj_bf16(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, plan, stream,
                       scratch.data_ptr() if scratch is not None else 0, scratch.numel() if scratch is not None else 0)
    return y


def _scratch_for(state: dict, m: int, n: int, k: int, plan) -> torch.Tensor | None:
    """The state's zeroed split-K scratch when the plan needs one (grown outside graph capture).

    One buffer serves every layer and shape of a state: split-K plans count contributors in its
    tile counters and park FP32 partials in it, so two projections of the same state must not run at
    the same time on different streams (their counters and partials would mix). Calls on one stream
    are ordered (a programmatic launch touches scratch only after its wait for the previous grid); a
    caller that serves one state from several streams at once needs one state per stream. The
    reference shares its split-K counters the same way (submission.py:1126)."""
    key = (m, n, k, plan.key())
    need = state["scratch_need"].get(key)
    if need is None:
        need = _lib.scratch_bytes(m, n, k, plan)
        state["scratch_need"][key] = need
    if need == 0:
        return None
    buf = state["scratch"]
    if buf is None or buf.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"split-K scratch of {need} bytes needed inside graph capture; call once before capturing")
        buf = torch.zeros(need, dtype=torch.uint8, device=state["scratch"].device if buf is not None else "cuda")
        state["scratch"] = buf
    return buf


def kernel_fn(data: Inputs, state) -> torch.Tensor:
    """data["x"] [m, k] BF16 @ W[:n].T -> [m, n] BF16 (FP32 for the router), for data["config"]["layer"].

    Launches on torch's current stream. One state's calls must not overlap in time on different
    streams: they share the state's split-K scratch (see _scratch_for)."""
    cfg = data["config"]
    return project(data["x"], state, cfg["layer"], cfg["n"])
