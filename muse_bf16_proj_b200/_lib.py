"""ctypes binding of libmuse_proj.so (the C ABI declared in include/muse_proj.h).

The library is built in-tree (``python -m muse_bf16_proj_b200.build``). There is no fallback:
if the library is missing or fails to load, every projection raises.
"""

from __future__ import annotations

import ctypes
import os
import re

from .build import LIB

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "muse_proj.h")

MUSE_OK = 0
ERRORS = {-1: "INVALID", -2: "ALIGN", -3: "SHAPE", -4: "CAPACITY", -5: "CUDA", -6: "TIMEOUT", -7: "PLAN"}
KERNEL_GEMV_BF16, KERNEL_GEMV_12B, KERNEL_TC_TILE, KERNEL_TC_STREAMK, KERNEL_TC_GEMM, KERNEL_TC_GEMM2 = 1, 2, 3, 4, 5, 6
KERNEL_TC_12B, KERNEL_TC_SKINNY, KERNEL_F32_GEMV, KERNEL_GEMV_12T, KERNEL_TC_ROWS, KERNEL_TC_WIDE = 7, 8, 9, 10, 11, 12
KERNEL_TC_PAIRK, KERNEL_GEMV_TILES = 13, 14
KERNEL_NAMES = {KERNEL_GEMV_BF16: "gemv_bf16", KERNEL_GEMV_12B: "gemv_12b", KERNEL_TC_TILE: "tc_tile",
                KERNEL_TC_STREAMK: "tc_streamk", KERNEL_TC_GEMM: "tc_gemm", KERNEL_TC_GEMM2: "tc_gemm2",
                KERNEL_TC_12B: "tc_12b", KERNEL_TC_SKINNY: "tc_skinny", KERNEL_F32_GEMV: "f32_gemv",
                KERNEL_GEMV_12T: "gemv_12t", KERNEL_TC_ROWS: "tc_rows", KERNEL_TC_WIDE: "tc_wide",
                KERNEL_TC_PAIRK: "tc_pairk", KERNEL_GEMV_TILES: "gemv_tiles"}
TILE_KERNELS = (KERNEL_TC_TILE, KERNEL_TC_STREAMK, KERNEL_TC_SKINNY, KERNEL_TC_GEMM, KERNEL_TC_GEMM2, KERNEL_TC_ROWS,
                KERNEL_TC_WIDE, KERNEL_TC_PAIRK, KERNEL_GEMV_TILES)
KERNEL_IDS = {v: k for k, v in KERNEL_NAMES.items()}
FLAG_GLOBAL_SPLIT = 1
FLAG_PDL = 2
FLAG_STREAMK = 4
FLAG_SK_TAIL = 8


class MuseError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"muse error {code} ({ERRORS.get(code, '?')}): {message}")
        self.code = code


class MusePlan(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in
                ("kernel", "split", "tile_n", "stages", "ctas", "warps", "chunk", "flags")]

    def as_dict(self) -> dict:
        d = {name: int(getattr(self, name)) for name, _ in self._fields_}
        d["kernel"] = KERNEL_NAMES.get(d["kernel"], d["kernel"])
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "MusePlan":
        p = cls()
        for name, _ in cls._fields_:
            v = d.get(name, 0)
            if name == "kernel" and isinstance(v, str):
                v = KERNEL_IDS[v]
            setattr(p, name, int(v))
        return p

    def key(self) -> tuple:
        return tuple(int(getattr(self, name)) for name, _ in self._fields_)


class MuseEnc12(ctypes.Structure):
    _fields_ = [("planes", ctypes.c_void_p), ("bases", ctypes.c_void_p), ("esc_ptr", ctypes.c_void_p),
                ("esc_val", ctypes.c_void_p), ("n", ctypes.c_int64), ("k", ctypes.c_int64), ("n_esc", ctypes.c_int64)]


MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class MuseGather(ctypes.Structure):
    """Mirror of include/muse_proj.h MuseGather: every rank's y_full and control block."""
    _fields_ = [("y", ctypes.c_void_p * MAX_PEERS), ("ctl", ctypes.c_void_p * MAX_PEERS), ("world", ctypes.c_int32),
                ("rank", ctypes.c_int32), ("ldy", ctypes.c_int64), ("col0", ctypes.c_int64)]


_lib = None

_P, _I64, _I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
_SIGNATURES = {
    "muse_version": ([], ctypes.c_char_p),
    "muse_last_error": ([], ctypes.c_char_p),
    "muse_sm_count": ([ctypes.POINTER(ctypes.c_int)], _I32),
    "muse_device_error": ([ctypes.POINTER(ctypes.c_int), _P], _I32),
    "muse_plan_default": ([_I64, _I64, _I64, _I32, ctypes.POINTER(MusePlan)], _I32),
    "muse_scratch_bytes": ([_I64, _I64, _I64, ctypes.POINTER(MusePlan), ctypes.POINTER(_I64)], _I32),
    "muse_proj_bf16": ([_P, _P, _P, _I64, _I64, _I64, ctypes.POINTER(MusePlan), _P, _I64, _P], _I32),
    "muse_tiles_bytes": ([_I64, _I64, ctypes.POINTER(_I64)], _I32),
    "muse_set_trace": ([_P, _I64], _I32),
    "muse_pack_tiles": ([_P, _P, _I64, _I64, _P], _I32),
    "muse_proj_bf16_tiles": ([_P, _P, _P, _I64, _I64, _I64, ctypes.POINTER(MusePlan), _P, _I64, _P], _I32),
    "muse_proj_12b": ([ctypes.POINTER(MuseEnc12), _P, _P, _I64, ctypes.POINTER(MusePlan), _P], _I32),
    "muse_tiles12_bytes": ([_I64, _I64, ctypes.POINTER(_I64)], _I32),
    "muse_pack_tiles12": ([ctypes.POINTER(MuseEnc12), _P, _P], _I32),
    "muse_proj_12b_tiles": ([ctypes.POINTER(MuseEnc12), _P, _P, _P, _I64, ctypes.POINTER(MusePlan), _P, _I64, _P], _I32),
    "muse_proj_bf16_tiles_f32": ([_P, _P, _P, _I64, _I64, _I64, ctypes.POINTER(MusePlan), _P, _I64, _P], _I32),
    "muse_router_tiles_bytes": ([_I64, _I64, ctypes.POINTER(_I64)], _I32),
    "muse_pack_router": ([_P, _P, _I64, _I64, _P], _I32),
    "muse_proj_f32": ([_P, _P, _P, _P, _I64, _I64, _I64, ctypes.POINTER(MusePlan), _P, _I64, _P], _I32),
    "muse_proj_bf16_tiles_noalloc": ([_P, _P, _P, _I64, _I64, _I64, ctypes.POINTER(MusePlan), _P], _I32),
    "muse_peer_ctl_bytes": ([ctypes.POINTER(_I64)], _I32),
    "muse_ipc_export": ([_P, _P, ctypes.POINTER(_I64)], _I32),
    "muse_ipc_open": ([_P, _I64, ctypes.POINTER(_P)], _I32),
    "muse_ipc_close": ([_P, _I64], _I32),
    "muse_proj_bf16_tiles_gather": ([_P, _P, _I64, _I64, _I64, ctypes.POINTER(MuseGather), ctypes.POINTER(MusePlan), _P,
                                     _I64, _P], _I32),
    "muse_encode12_sizes": ([_I64, _I64, ctypes.POINTER(_I64), ctypes.POINTER(_I64)], _I32),
    "muse_encode12": ([_P, _I64, _I64, _P, _P, _P, _P, _I64, ctypes.POINTER(_I64), _I32], _I32),
    "muse_encode12_device": ([_P, _I64, _I64, _P, _P, _P, _P], _I32),
    "muse_encode12_device_escapes": ([_P, _I64, _I64, _P, _P, _P, _I64, _P], _I32),
    "muse_decode12": ([_P, _P, _P, _P, _I64, _I64, _P, _I32], _I32),
    "muse_stream_read": ([_P, _I64, _I64, _I32, _I32, _P, _P], _I32),
    "muse_rows_groups": ([_I64, _I64, _I64, ctypes.POINTER(MusePlan), ctypes.POINTER(ctypes.c_int)], _I32),
    "muse_rows_bytes": ([_I64, _I64, _I32, ctypes.POINTER(_I64)], _I32),
    "muse_pack_rows": ([_P, _P, _I64, _I64, _I32, _P], _I32),
    "muse_proj_bf16_rows": ([_P, _P, _P, _I64, _I64, _I64, ctypes.POINTER(MusePlan), _P], _I32),
}


def declared_symbols() -> list[str]:
    """Function names declared in include/muse_proj.h."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(muse_\w+)\s*\(", text, flags=re.M)))


def load():
    """The loaded library (loads it on first use). Raises if it is not built."""
    global _lib
    if _lib is None:
        path = os.environ.get("MUSE_PROJ_LIB", LIB)
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is not built: run `python -m muse_bf16_proj_b200.build` (no fallback path exists)")
        lib = ctypes.CDLL(path)
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def check(rc: int) -> None:
    if rc != MUSE_OK:
        raise MuseError(rc, load().muse_last_error().decode(errors="replace"))


def version() -> str:
    return load().muse_version().decode()


def sm_count() -> int:
    out = ctypes.c_int()
    check(load().muse_sm_count(ctypes.byref(out)))
    return out.value


def device_error(stream: int = 0) -> int:
    """The device error word (0 = none), cleared afterwards. Raises MuseError when it was set."""
    code = ctypes.c_int()
    rc = load().muse_device_error(ctypes.byref(code), ctypes.c_void_p(stream))
    if rc != MUSE_OK:
        raise MuseError(rc, load().muse_last_error().decode(errors="replace"))
    return code.value


WEIGHTS_ROW_MAJOR, WEIGHTS_12B, WEIGHTS_TILES, WEIGHTS_12B_TILES, WEIGHTS_F32 = 0, 1, 2, 3, 4


def plan_default(m: int, n: int, k: int, weights_12b: bool = False, tiles: bool = False, f32: bool = False) -> MusePlan:
    """The library's default plan; weights_12b with tiles means the 12-bit tiles (GEMV_12T up to 4
    tokens, TC_12B above); f32: the router's FP32 W with its hi | lo tiles."""
    p = MusePlan()
    if f32:
        fmt = WEIGHTS_F32
    elif weights_12b:
        fmt = WEIGHTS_12B_TILES if tiles else WEIGHTS_12B
    else:
        fmt = WEIGHTS_TILES if tiles else WEIGHTS_ROW_MAJOR
    check(load().muse_plan_default(m, n, k, fmt, ctypes.byref(p)))
    return p


def proj_bf16(x_ptr: int, w_ptr: int, y_ptr: int, m: int, n: int, k: int, plan: MusePlan, stream: int,
              scratch_ptr: int = 0, scratch_bytes: int = 0) -> None:
    check(load().muse_proj_bf16(x_ptr, w_ptr, y_ptr, m, n, k, ctypes.byref(plan), scratch_ptr or None, scratch_bytes,
                                ctypes.c_void_p(stream)))


def proj_bf16_tiles(x_ptr: int, tiles_ptr: int, y_ptr: int, m: int, n: int, k: int, plan: MusePlan, stream: int,
                    scratch_ptr: int = 0, scratch_bytes: int = 0) -> None:
    check(load().muse_proj_bf16_tiles(x_ptr, tiles_ptr, y_ptr, m, n, k, ctypes.byref(plan), scratch_ptr or None,
                                      scratch_bytes, ctypes.c_void_p(stream)))


def scratch_bytes(m: int, n: int, k: int, plan: MusePlan) -> int:
    out = ctypes.c_int64()
    check(load().muse_scratch_bytes(m, n, k, ctypes.byref(plan), ctypes.byref(out)))
    return out.value


def tiles_bytes(n: int, k: int) -> int:
    out = ctypes.c_int64()
    check(load().muse_tiles_bytes(n, k, ctypes.byref(out)))
    return out.value


def pack_tiles(w_ptr: int, tiles_ptr: int, n: int, k: int, stream: int) -> None:
    check(load().muse_pack_tiles(w_ptr, tiles_ptr, n, k, ctypes.c_void_p(stream)))


def proj_12b(enc: MuseEnc12, x_ptr: int, y_ptr: int, m: int, plan: MusePlan, stream: int) -> None:
    check(load().muse_proj_12b(ctypes.byref(enc), x_ptr, y_ptr, m, ctypes.byref(plan), ctypes.c_void_p(stream)))


def tiles12_bytes(n: int, k: int) -> int:
    out = ctypes.c_int64()
    check(load().muse_tiles12_bytes(n, k, ctypes.byref(out)))
    return out.value


def pack_tiles12(enc: MuseEnc12, tiles12_ptr: int, stream: int) -> None:
    check(load().muse_pack_tiles12(ctypes.byref(enc), tiles12_ptr, ctypes.c_void_p(stream)))


def encode12_device(w_ptr: int, n: int, k: int, planes_ptr: int, bases_ptr: int, esc_ptr_ptr: int,
                    stream: int) -> None:
    """Step 1 of the device encoder (planes, bases, esc_ptr); all device pointers."""
    check(load().muse_encode12_device(w_ptr, n, k, planes_ptr, bases_ptr, esc_ptr_ptr, ctypes.c_void_p(stream)))


def encode12_device_escapes(w_ptr: int, n: int, k: int, bases_ptr: int, esc_ptr_ptr: int, esc_val_ptr: int,
                            esc_cap: int, stream: int) -> None:
    """Step 2 of the device encoder: the escape entries into esc_val[esc_cap]."""
    check(load().muse_encode12_device_escapes(w_ptr, n, k, bases_ptr, esc_ptr_ptr, esc_val_ptr or None, esc_cap,
                                              ctypes.c_void_p(stream)))


def proj_12b_tiles(enc: MuseEnc12, tiles12_ptr: int, x_ptr: int, y_ptr: int, m: int, plan: MusePlan, stream: int,
                   scratch_ptr: int = 0, scratch_bytes: int = 0) -> None:
    check(load().muse_proj_12b_tiles(ctypes.byref(enc), tiles12_ptr, x_ptr, y_ptr, m, ctypes.byref(plan),
                                     scratch_ptr or None, scratch_bytes, ctypes.c_void_p(stream)))


def proj_bf16_tiles_f32(x_ptr: int, tiles_ptr: int, y_ptr: int, m: int, n: int, k: int, plan: MusePlan, stream: int,
                        scratch_ptr: int = 0, scratch_bytes: int = 0) -> None:
    check(load().muse_proj_bf16_tiles_f32(x_ptr, tiles_ptr, y_ptr, m, n, k, ctypes.byref(plan), scratch_ptr or None,
                                          scratch_bytes, ctypes.c_void_p(stream)))


def router_tiles_bytes(n: int, k: int) -> int:
    out = ctypes.c_int64()
    check(load().muse_router_tiles_bytes(n, k, ctypes.byref(out)))
    return out.value


def pack_router(w_ptr: int, tiles_ptr: int, n: int, k: int, stream: int) -> None:
    check(load().muse_pack_router(w_ptr, tiles_ptr, n, k, ctypes.c_void_p(stream)))


def proj_f32(x_ptr: int, w_ptr: int, tiles_ptr: int, y_ptr: int, m: int, n: int, k: int, plan: MusePlan, stream: int,
             scratch_ptr: int = 0, scratch_bytes: int = 0) -> None:
    check(load().muse_proj_f32(x_ptr, w_ptr or None, tiles_ptr or None, y_ptr, m, n, k, ctypes.byref(plan),
                               scratch_ptr or None, scratch_bytes, ctypes.c_void_p(stream)))


def peer_ctl_bytes() -> int:
    out = ctypes.c_int64()
    check(load().muse_peer_ctl_bytes(ctypes.byref(out)))
    return out.value


def ipc_export(ptr: int) -> tuple[bytes, int]:
    """(CUDA IPC handle of the allocation holding device pointer `ptr`, ptr's offset in it)."""
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    off = ctypes.c_int64()
    check(load().muse_ipc_export(ptr, handle, ctypes.byref(off)))
    return handle.raw, off.value


def ipc_open(handle: bytes, offset: int) -> int:
    """A peer process's exported device pointer, opened in this process."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError(f"an IPC handle is {IPC_HANDLE_BYTES} bytes (got {len(handle)})")
    out = ctypes.c_void_p()
    check(load().muse_ipc_open(handle, offset, ctypes.byref(out)))
    return out.value


def ipc_close(ptr: int, offset: int) -> None:
    check(load().muse_ipc_close(ptr, offset))


def proj_bf16_tiles_gather(x_ptr: int, tiles_ptr: int, m: int, n: int, k: int, gather: MuseGather, plan: MusePlan,
                           stream: int, scratch_ptr: int = 0, scratch_bytes: int = 0) -> None:
    check(load().muse_proj_bf16_tiles_gather(x_ptr, tiles_ptr, m, n, k, ctypes.byref(gather), ctypes.byref(plan),
                                             scratch_ptr or None, scratch_bytes, ctypes.c_void_p(stream)))


TRACE_RECORD_BYTES = 64


def set_trace(ptr: int, capacity: int) -> None:
    """Per-CTA timestamps for later launches into a device buffer (ptr 0 turns tracing off)."""
    check(load().muse_set_trace(ptr or None, capacity))


NOALLOC_SCRATCH_BYTES = 8 * 1024 * 1024


def proj_bf16_tiles_noalloc(x_ptr: int, tiles_ptr: int, y_ptr: int, m: int, n: int, k: int, plan: MusePlan,
                            stream: int) -> None:
    """muse_proj_bf16_tiles_noalloc: the stream-K projection with the library's built-in scratch
    (for callers that cannot allocate device memory); see include/muse_proj.h."""
    check(load().muse_proj_bf16_tiles_noalloc(x_ptr, tiles_ptr, y_ptr, m, n, k, ctypes.byref(plan),
                                              ctypes.c_void_p(stream)))


def stream_read(src_ptr: int, nbytes: int, chunk: int, stages: int, ctas: int, count_ptr: int, stream: int) -> None:
    """muse_stream_read: the bulk-copy streaming-read floor over nbytes at src_ptr; adds the chunks
    that landed to the device u32 at count_ptr."""
    check(load().muse_stream_read(src_ptr, nbytes, chunk, stages, ctas, count_ptr, ctypes.c_void_p(stream)))


def rows_groups(m: int, n: int, k: int, plan: MusePlan) -> int:
    """Row windows of a TC_ROWS plan at this shape (the groups of its window-major weight copy)."""
    out = ctypes.c_int()
    check(load().muse_rows_groups(m, n, k, ctypes.byref(plan), ctypes.byref(out)))
    return out.value


def rows_bytes(n: int, k: int, groups: int) -> int:
    out = ctypes.c_int64()
    check(load().muse_rows_bytes(n, k, groups, ctypes.byref(out)))
    return out.value


def pack_rows(w_ptr: int, out_ptr: int, n: int, k: int, groups: int, stream: int) -> None:
    check(load().muse_pack_rows(w_ptr, out_ptr, n, k, groups, ctypes.c_void_p(stream)))


def proj_bf16_rows(x_ptr: int, wrows_ptr: int, y_ptr: int, m: int, n: int, k: int, plan: MusePlan, stream: int) -> None:
    check(load().muse_proj_bf16_rows(x_ptr, wrows_ptr, y_ptr, m, n, k, ctypes.byref(plan), ctypes.c_void_p(stream)))
