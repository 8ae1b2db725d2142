"""ctypes binding of libad_b200.so (declared in include/ad_b200.h).

Loads the in-tree library; fails loudly when it is missing (no CPU fallback).
"""
import ctypes
import hashlib
import os
import threading
from typing import Dict, List, Optional, Sequence

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libad_b200.so")

_lib = None
_lock = threading.Lock()

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_uint = ctypes.c_uint
c_size_t = ctypes.c_size_t
c_u64 = ctypes.c_uint64
c_u32 = ctypes.c_uint32
c_char_p = ctypes.c_char_p

# name -> (restype, argtypes); must match include/ad_b200.h
SIGNATURES = {
    "ad_version": (c_int, []),
    "ad_last_error": (c_char_p, []),
    "ad_device_count": (c_int, [ctypes.POINTER(c_int)]),
    "ad_init": (c_int, [c_int, c_int, ctypes.POINTER(c_void_p)]),
    "ad_destroy": (c_int, [c_void_p]),
    "ad_device_info": (c_int, [c_void_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                               ctypes.POINTER(c_size_t), ctypes.POINTER(c_size_t)]),
    "ad_malloc": (c_int, [c_void_p, c_size_t, ctypes.POINTER(c_u64)]),
    "ad_free": (c_int, [c_void_p, c_u64]),
    "ad_memset": (c_int, [c_void_p, c_u64, c_int, c_size_t, c_int]),
    "ad_pinned_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p)]),
    "ad_pinned_free": (c_int, [c_void_p]),
    "ad_h2d": (c_int, [c_void_p, c_u64, c_void_p, c_size_t, c_int]),
    "ad_d2h": (c_int, [c_void_p, c_void_p, c_u64, c_size_t, c_int]),
    "ad_d2d": (c_int, [c_void_p, c_u64, c_u64, c_size_t, c_int]),
    "ad_h2d_pageable": (c_int, [c_void_p, c_u64, c_void_p, c_size_t, c_int]),
    "ad_d2h_pageable": (c_int, [c_void_p, c_void_p, c_u64, c_size_t, c_int]),
    "ad_host_copy": (c_int, [c_void_p, c_void_p, c_size_t]),
    "ad_stream_sync": (c_int, [c_void_p, c_int]),
    "ad_sync": (c_int, [c_void_p]),
    "ad_event_create": (c_int, [c_void_p, c_int, ctypes.POINTER(c_void_p)]),
    "ad_event_destroy": (c_int, [c_void_p]),
    "ad_event_record": (c_int, [c_void_p, c_void_p, c_int]),
    "ad_stream_wait_event": (c_int, [c_void_p, c_int, c_void_p]),
    "ad_event_sync": (c_int, [c_void_p]),
    "ad_event_elapsed_ms": (c_int, [c_void_p, c_void_p, ctypes.POINTER(ctypes.c_float)]),
    "ad_compile_cubin": (c_int, [c_char_p, c_char_p, ctypes.POINTER(c_char_p), c_int,
                                 ctypes.POINTER(c_void_p), ctypes.POINTER(c_size_t), c_char_p, c_size_t]),
    "ad_free_host": (None, [c_void_p]),
    "ad_load_kernel": (c_int, [c_void_p, c_void_p, c_char_p, ctypes.POINTER(c_void_p)]),
    "ad_kernel_free": (c_int, [c_void_p]),
    "ad_kernel_set_smem": (c_int, [c_void_p, c_int]),
    "ad_kernel_attr": (c_int, [c_void_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "ad_launch": (c_int, [c_void_p, c_void_p, c_uint, c_uint, c_uint, c_uint, c_uint, c_uint, c_uint,
                          ctypes.POINTER(c_void_p), c_int]),
    "ad_check": (c_int, [c_void_p]),
    "ad_tmap_2d": (c_int, [c_u64, c_u64, c_u64, c_u64, c_u32, c_u32, c_int, c_int, c_void_p]),
    "ad_graph_begin": (c_int, [c_void_p, c_int]),
    "ad_graph_end": (c_int, [c_void_p, c_int, ctypes.POINTER(c_void_p)]),
    "ad_graph_launch": (c_int, [c_void_p, c_void_p, c_int]),
    "ad_graph_destroy": (c_int, [c_void_p]),
    "ad_nccl_unique_id": (c_int, [c_void_p]),
    "ad_nccl_init": (c_int, [c_void_p, c_int, c_int, c_void_p, ctypes.c_double]),
    "ad_allreduce_f32": (c_int, [c_void_p, c_u64, c_u64, c_size_t, c_int, c_int]),
    "ad_nccl_abort": (c_int, [c_void_p]),
    "ad_peer_init": (c_int, [c_void_p, c_u64, c_size_t]),
    "ad_peer_allreduce_f32": (c_int, [c_void_p, c_u64, c_size_t, c_int, c_int, c_u64]),
    "ad_peer_close": (c_int, [c_void_p]),
    "ad_profiler_range": (c_int, [c_int]),
    "ad_dot_tf32x3_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
}


class ADError(RuntimeError):
    pass


def lib():
    """The loaded library (built on first use if the sources are newer)."""
    global _lib
    with _lock:
        if _lib is None:
            from . import build as _build
            if _build.needs_build():
                _build.build()
            if not os.path.exists(LIB_PATH):
                raise ADError(f"{LIB_PATH} missing: the CUDA backend is not built")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
        return _lib


def check(status: int, what: str = "") -> None:
    if status != 0:
        msg = lib().ad_last_error().decode(errors="replace")
        raise ADError(f"{what}: {msg}" if what else msg)


# ------------------------------------------------------------------ NVRTC compile cache

CACHE_DIR = os.environ.get("AD_B200_CACHE", os.path.join(os.path.expanduser("~"), ".cache", "ad_b200"))
_mem_cache: Dict[str, bytes] = {}

NVRTC_OPTS = ["--gpu-architecture=sm_100a", "-std=c++17", "-default-device", "-lineinfo",
              "--extra-device-vectorization"]


def compile_cubin(src: str, name: str = "k.cu", opts: Optional[Sequence[str]] = None) -> bytes:
    """NVRTC -> sm_100a cubin, cached in memory and on disk by source hash."""
    opts = list(opts) if opts is not None else list(NVRTC_OPTS)
    key = hashlib.sha256(("\0".join(opts) + "\0" + src).encode()).hexdigest()[:32]
    if key in _mem_cache:
        return _mem_cache[key]
    path = os.path.join(CACHE_DIR, key + ".cubin")
    if os.path.exists(path):
        with open(path, "rb") as f:
            data = f.read()
        _mem_cache[key] = data
        return data
    L = lib()
    arr = (c_char_p * len(opts))(*[o.encode() for o in opts])
    out = c_void_p()
    size = c_size_t()
    log = ctypes.create_string_buffer(8192)
    check(L.ad_compile_cubin(src.encode(), name.encode(), arr, len(opts), ctypes.byref(out),
                             ctypes.byref(size), log, 8192), f"compile {name}")
    data = ctypes.string_at(out, size.value)
    L.ad_free_host(out)
    try:
        os.makedirs(CACHE_DIR, exist_ok=True)
        tmp = f"{path}.{os.getpid()}.{threading.get_ident()}"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    except OSError:
        pass
    _mem_cache[key] = data
    return data


# ------------------------------------------------------------------ context wrapper

def host_copy(dst_ptr: int, src_ptr: int, nbytes: int) -> None:
    """memcpy on the library's copy threads."""
    check(lib().ad_host_copy(dst_ptr, src_ptr, nbytes), "ad_host_copy")


class Context:
    """One device context: streams, memory, kernels (C-ABI ``ad_ctx``)."""

    COMPUTE, H2D, D2H, COMM = 0, 1, 2, 3

    def __init__(self, device: int = 0, n_streams: int = 4):
        self.L = lib()
        h = c_void_p()
        check(self.L.ad_init(device, n_streams, ctypes.byref(h)), f"ad_init(device={device})")
        self.h = h
        self.device = device
        sm = c_int()
        smem = c_int()
        fb = c_size_t()
        tb = c_size_t()
        check(self.L.ad_device_info(h, ctypes.byref(sm), ctypes.byref(smem), ctypes.byref(fb), ctypes.byref(tb)))
        self.sm_count = sm.value
        self.smem_optin = smem.value
        self.total_bytes = tb.value

    def free_bytes(self) -> int:
        fb = c_size_t()
        check(self.L.ad_device_info(self.h, None, None, ctypes.byref(fb), None))
        return fb.value

    def malloc(self, nbytes: int) -> int:
        p = c_u64()
        check(self.L.ad_malloc(self.h, nbytes, ctypes.byref(p)), f"ad_malloc({nbytes})")
        return p.value

    def free(self, p: int) -> None:
        check(self.L.ad_free(self.h, p), "ad_free")

    def memset(self, p: int, value: int, nbytes: int, stream: int = 0) -> None:
        check(self.L.ad_memset(self.h, p, value, nbytes, stream), "ad_memset")

    def h2d(self, dst: int, src_ptr: int, nbytes: int, stream: int = 0) -> None:
        check(self.L.ad_h2d(self.h, dst, src_ptr, nbytes, stream), "ad_h2d")

    def d2h(self, dst_ptr: int, src: int, nbytes: int, stream: int = 0) -> None:
        check(self.L.ad_d2h(self.h, dst_ptr, src, nbytes, stream), "ad_d2h")

    def h2d_pageable(self, dst: int, src_ptr: int, nbytes: int, stream: int = 0) -> None:
        """From pageable host memory; ``src`` may be reused on return."""
        check(self.L.ad_h2d_pageable(self.h, dst, src_ptr, nbytes, stream), "ad_h2d_pageable")

    def d2h_pageable(self, dst_ptr: int, src: int, nbytes: int, stream: int = 0) -> None:
        """Into pageable host memory; complete on return."""
        check(self.L.ad_d2h_pageable(self.h, dst_ptr, src, nbytes, stream), "ad_d2h_pageable")

    def d2d(self, dst: int, src: int, nbytes: int, stream: int = 0) -> None:
        check(self.L.ad_d2d(self.h, dst, src, nbytes, stream), "ad_d2d")

    def sync(self, stream: Optional[int] = None) -> None:
        if stream is None:
            check(self.L.ad_sync(self.h), "ad_sync")
        else:
            check(self.L.ad_stream_sync(self.h, stream), "ad_stream_sync")

    def event(self, timing: bool = False) -> "Event":
        return Event(self, timing)

    def load(self, cubin: bytes, fn: str) -> "Kernel":
        return Kernel(self, cubin, fn)

    def launch(self, k: "Kernel", grid, block, smem: int, args, stream: int = 0) -> None:
        gx, gy, gz = (tuple(grid) + (1, 1))[:3]
        bx, by, bz = (tuple(block) + (1, 1))[:3]
        check(self.L.ad_launch(self.h, k.h, gx, gy, gz, bx, by, bz, smem, args, stream), "ad_launch")

    def close(self) -> None:
        if self.h:
            self.L.ad_destroy(self.h)
            self.h = None


class Event:
    def __init__(self, ctx: Context, timing: bool):
        self.ctx = ctx
        h = c_void_p()
        check(ctx.L.ad_event_create(ctx.h, int(timing), ctypes.byref(h)), "ad_event_create")
        self.h = h

    def record(self, stream: int = 0) -> None:
        check(self.ctx.L.ad_event_record(self.ctx.h, self.h, stream), "ad_event_record")

    def wait_on(self, stream: int) -> None:
        """Make ``stream`` wait for this event."""
        check(self.ctx.L.ad_stream_wait_event(self.ctx.h, stream, self.h), "ad_stream_wait_event")

    def sync(self) -> None:
        check(self.ctx.L.ad_event_sync(self.h), "ad_event_sync")

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float()
        check(self.ctx.L.ad_event_elapsed_ms(self.h, end.h, ctypes.byref(ms)), "ad_event_elapsed_ms")
        return ms.value

    def __del__(self):
        try:
            if self.h:
                self.ctx.L.ad_event_destroy(self.h)
        except Exception:
            pass


class Kernel:
    def __init__(self, ctx: Context, cubin: bytes, fn: str):
        self.ctx = ctx
        h = c_void_p()
        buf = ctypes.create_string_buffer(cubin, len(cubin))
        check(ctx.L.ad_load_kernel(ctx.h, buf, fn.encode(), ctypes.byref(h)), f"load {fn}")
        self.h = h
        self.name = fn
        self.smem = 0

    def set_smem(self, nbytes: int) -> None:
        check(self.ctx.L.ad_kernel_set_smem(self.h, nbytes), "ad_kernel_set_smem")
        self.smem = nbytes

    def attrs(self):
        r, s, t = c_int(), c_int(), c_int()
        check(self.ctx.L.ad_kernel_attr(self.h, ctypes.byref(r), ctypes.byref(s), ctypes.byref(t)))
        return {"regs": r.value, "static_smem": s.value, "max_threads": t.value}


def tmap_2d(base: int, rows: int, cols: int, row_stride_bytes: int, box_rows: int, box_cols: int,
            elem_bytes: int = 4, swizzle: int = 128) -> bytes:
    out = ctypes.create_string_buffer(128)
    check(lib().ad_tmap_2d(base, rows, cols, row_stride_bytes, box_rows, box_cols, elem_bytes,
                           swizzle, out), "ad_tmap_2d")
    return out.raw


class Graph:
    def __init__(self, ctx: Context, h):
        self.ctx = ctx
        self.h = h

    def launch(self, stream: int = 0) -> None:
        check(self.ctx.L.ad_graph_launch(self.ctx.h, self.h, stream), "ad_graph_launch")

    def __del__(self):
        try:
            self.ctx.L.ad_graph_destroy(self.h)
        except Exception:
            pass


def graph_begin(ctx: Context, stream: int = 0) -> None:
    check(ctx.L.ad_graph_begin(ctx.h, stream), "ad_graph_begin")


def graph_end(ctx: Context, stream: int = 0) -> Graph:
    h = c_void_p()
    check(ctx.L.ad_graph_end(ctx.h, stream, ctypes.byref(h)), "ad_graph_end")
    return Graph(ctx, h)


def device_count() -> int:
    n = c_int()
    if lib().ad_device_count(ctypes.byref(n)) != 0:
        return 0
    return n.value
