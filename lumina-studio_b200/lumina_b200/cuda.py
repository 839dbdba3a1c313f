"""ctypes boundary to liblumina_cuda.so (the B200 Lumina decode path).

Same contract as the reference's ``tops.py`` (src/lumina_framework/tops.py):

  * the library is located (``LUMINA_CUDA_LIB`` or the in-tree build next to
    this file), bound once under a lock (tops.py:264-270), its version must
    equal ``VERSION`` (tops.py:95-97) and a numeric self-test must pass on
    the device before it is trusted (tops.py:152-261);
  * ``LUMINA_CUDA_DISABLE=1`` forces unavailable (tops.py:242);
  * the tops-style functions (``gemv_int8``, ``gemv_q4_0``, ``gemv_fp16``,
    ``gemm_int8``) return ``{"out": array}`` or ``{"error": reason}`` and
    never raise (tops.py:296-420).

Unlike the reference there is no CPU fallback behind any of these calls: if
the CUDA library is unavailable the caller gets the error, and the model
classes built on top raise.
"""
from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
VERSION = 1

LUMINA_OK = 0
ERRORS = {1: "bad argument", 2: "cuda error", 3: "unsupported", 4: "out of device memory",
          5: "bad state", 6: "nccl error", 7: "self-test mismatch"}
KIND_BITS = {"int4": 4, "int3": 3, "int2": 2, "binary": 1}
PACK = {"none": 0, "nibble": 1, "2bit": 2}

_STATE: dict | None = None
_LOCK = threading.Lock()
_SELFTESTED: set[int] = set()


class LuminaError(RuntimeError):
    def __init__(self, code: int, text: str):
        super().__init__("%s (%d): %s" % (ERRORS.get(code, "error"), code, text))
        self.code = code


class ModelConfig(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_int), ("d_model", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn", ctypes.c_int),
                ("vocab", ctypes.c_int), ("eps", ctypes.c_float), ("theta", ctypes.c_float),
                ("kv_fp16", ctypes.c_int), ("block_size", ctypes.c_int), ("max_seq", ctypes.c_int),
                ("max_rows", ctypes.c_int), ("tp_rank", ctypes.c_int), ("tp_size", ctypes.c_int)]


def lib_path() -> str:
    return os.environ.get("LUMINA_CUDA_LIB") or os.path.join(HERE, "liblumina_cuda.so")


_VP = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_FP = ctypes.POINTER(ctypes.c_float)
_IP = ctypes.POINTER(ctypes.c_int)
_U8P = ctypes.POINTER(ctypes.c_uint8)
_I8P = ctypes.POINTER(ctypes.c_int8)

# name -> argtypes; every entry returns int (status) unless listed in _RESTYPE
SIGNATURES = {
    "lumina_cuda_version": [],
    "lumina_last_error": [],
    "lumina_device_count": [_IP],
    "lumina_selftest": [_I],
    "lumina_weight_upload": [_I, _I, _I, _I, _U8P, _SZ, _FP, _SZ, _I, _I, ctypes.POINTER(_VP)],
    "lumina_weight_free": [_VP],
    "lumina_weight_info": [_VP, _IP, _IP, _IP, _IP, ctypes.POINTER(_SZ), _IP],
    "lumina_weight_unpack": [_VP, _VP, _VP],
    "lumina_weight_dequant": [_VP, _VP, _VP],
    "lumina_gemv": [_VP, _VP, _I, _I, _VP, _I, _VP],
    "lumina_gemv_host": [_VP, _FP, _I, _FP],
    "lumina_gemv_noalloc": [_VP, _VP, _I, _I, _VP, _I, _VP],
    "lumina_gemm_rows": [_VP, _VP, _I, _I, _VP, _I, _VP],
    "lumina_gemv_int8": [_I8P, _FP, _I8P, _FP, _FP, _I, _I],
    "lumina_gemv_q4_0": [_I8P, _FP, _U8P, _FP, _FP, _I, _I],
    "lumina_gemv_fp16": [_VP, _VP, _FP, _I, _I],
    "lumina_gemm_int8": [_I8P, _FP, _I8P, _FP, _FP, _I, _I, _I],
    "lumina_model_create": [_I, ctypes.POINTER(ModelConfig), ctypes.POINTER(_VP)],
    "lumina_model_set_weight": [_VP, ctypes.c_char_p, _VP],
    "lumina_model_set_tensor": [_VP, ctypes.c_char_p, _FP, _I, _I],
    "lumina_model_set_moe": [_VP, _I, _I, _I, _I],
    "lumina_model_finalize": [_VP],
    "lumina_model_free": [_VP],
    "lumina_model_peer_handle": [_VP, _U8P],
    "lumina_model_init_peers": [_VP, _U8P],
    "lumina_kv_length": [_VP, _I, _IP],
    "lumina_kv_truncate": [_VP, _I],
    "lumina_kv_read": [_VP, _I, _I, _I, _FP, _FP],
    "lumina_kv_commit_rows": [_VP, _I, _IP, _I],
    "lumina_layer_forward": [_VP, _I, _VP, _I, _I, _IP, _FP, _VP],
    "lumina_forward": [_VP, _IP, _I, _I, _IP, _FP, _FP, _I],
    "lumina_decode_step": [_VP, _I, _FP, _IP],
    "lumina_decode_greedy": [_VP, _I, _I, _IP, _FP, _IP],
    "lumina_profile_gemv": [_VP, _I, _FP, _IP, ctypes.POINTER(ctypes.c_double)],
    "lumina_kv_attend": [_VP, _I, _FP, _FP],
    "lumina_profile_attention": [_VP, _I, _FP, ctypes.POINTER(ctypes.c_double)],
    "lumina_fault_status": [_I, _IP, _I],
    "lumina_debug_wait_limit": [ctypes.c_longlong],
}
_RESTYPE = {"lumina_last_error": ctypes.c_char_p}


def _bind(path: str) -> ctypes.CDLL:
    lib = ctypes.CDLL(path)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, ctypes.c_int)
    if int(lib.lumina_cuda_version()) != VERSION:
        raise RuntimeError("liblumina_cuda version mismatch")
    return lib


def _init() -> dict:
    if os.environ.get("LUMINA_CUDA_DISABLE") == "1":
        return {"ok": False, "reason": "disabled by LUMINA_CUDA_DISABLE=1"}
    path = lib_path()
    if not os.path.exists(path):
        return {"ok": False, "reason": "library not built: " + path}
    try:
        lib = _bind(path)
    except Exception as e:  # noqa: BLE001
        return {"ok": False, "reason": "%s: %s" % (type(e).__name__, str(e)[:160])}
    n = ctypes.c_int(0)
    if lib.lumina_device_count(ctypes.byref(n)) != 0 or n.value < 1:
        return {"ok": False, "reason": "no CUDA device", "path": path, "lib": lib, "bound": True}
    return {"ok": True, "path": path, "lib": lib, "bound": True, "devices": n.value,
            "reason": "bound"}


def state() -> dict:
    global _STATE
    if _STATE is None:
        with _LOCK:
            if _STATE is None:
                _STATE = _init()
    return _STATE


def bound_lib() -> ctypes.CDLL:
    """The bound library even without a device (symbol checks on CPU)."""
    s = state()
    if not s.get("bound"):
        raise LuminaError(2, s.get("reason", "unavailable"))
    return s["lib"]


def ensure_device(device: int = 0) -> ctypes.CDLL:
    """Library handle after the self-test passed on ``device``; raises."""
    s = state()
    if not s.get("ok"):
        raise LuminaError(2, "liblumina_cuda unavailable: " + str(s.get("reason")))
    lib = s["lib"]
    if device not in _SELFTESTED:
        with _LOCK:
            if device not in _SELFTESTED:
                rc = lib.lumina_selftest(device)
                if rc != 0:
                    raise LuminaError(rc, last_error(lib))
                _SELFTESTED.add(device)
    return lib


def available(device: int = 0) -> bool:
    try:
        ensure_device(device)
        return True
    except Exception:  # noqa: BLE001
        return False


def reason() -> str:
    s = state()
    return ("available: " if s.get("ok") else "unavailable: ") + str(s.get("reason"))


def info() -> dict:
    s = state()
    return {"available": bool(s.get("ok")), "reason": s.get("reason"), "path": s.get("path"),
            "version": VERSION, "devices": s.get("devices", 0),
            "disabled_env": os.environ.get("LUMINA_CUDA_DISABLE")}


def last_error(lib=None) -> str:
    lib = lib or bound_lib()
    v = lib.lumina_last_error()
    return v.decode() if v else ""


def check(rc: int, lib=None) -> None:
    if rc != 0:
        raise LuminaError(rc, last_error(lib))


def ptr(arr: np.ndarray, ctype):
    return arr.ctypes.data_as(ctypes.POINTER(ctype))


def fault_status(device: int = 0, clear: bool = True) -> int:
    """The device's fault word after its queued work finished (non-zero: a
    bounded wait inside an asynchronous GEMV gave up; see lumina_gemv)."""
    lib = bound_lib()
    w = ctypes.c_int(0)
    check(lib.lumina_fault_status(int(device), ctypes.byref(w), 1 if clear else 0), lib)
    return w.value


def debug_wait_limit(spins: int) -> None:
    """Testing aid: polls before a kernel's wait on a pending transfer gives
    up (0 = at once, negative = the default of about a second)."""
    check(bound_lib().lumina_debug_wait_limit(int(spins)))


# ---------------------------------------------------------------------------
# packed weights
# ---------------------------------------------------------------------------
class Weight:
    """A packed Lumina tensor resident on one device."""

    def __init__(self, handle, device, kind, rows, cols, group):
        self.handle, self.device = handle, device
        self.kind, self.rows, self.cols, self.group = kind, rows, cols, group
        self._owned = True

    @classmethod
    def upload(cls, kind: str, group: int, pack: str, codes: np.ndarray, scales: np.ndarray,
               rows: int, cols: int, device: int = 0) -> "Weight":
        lib = ensure_device(device)
        codes = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1)
        scales = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
        h = ctypes.c_void_p()
        check(lib.lumina_weight_upload(device, KIND_BITS[kind], int(group), PACK[pack],
                                       ptr(codes, ctypes.c_uint8), codes.size,
                                       ptr(scales, ctypes.c_float), scales.size,
                                       int(rows), int(cols), ctypes.byref(h)), lib)
        return cls(h, device, kind, rows, cols, group)

    def release(self):
        """Hand ownership to a model (lumina_model_set_weight)."""
        self._owned = False
        return self.handle

    def free(self):
        """Free the device copy now (queued work that reads it must be done)."""
        if self._owned and self.handle:
            check(bound_lib().lumina_weight_free(self.handle))
        self.handle = None

    def info(self) -> dict:
        lib = bound_lib()
        k, g, r, c, f = (ctypes.c_int() for _ in range(5))
        b = ctypes.c_size_t()
        check(lib.lumina_weight_info(self.handle, *(ctypes.byref(v) for v in (k, g, r, c)),
                                     ctypes.byref(b), ctypes.byref(f)), lib)
        return {"bits": k.value, "group": g.value, "rows": r.value, "cols": c.value,
                "device_bytes": b.value, "fp16_scales": bool(f.value)}

    def unpack(self, out_dev_ptr: int, stream: int = 0):
        check(bound_lib().lumina_weight_unpack(self.handle, out_dev_ptr, stream))

    def dequant(self, out_dev_ptr: int, stream: int = 0):
        check(bound_lib().lumina_weight_dequant(self.handle, out_dev_ptr, stream))

    def gemv(self, x_dev: int, batch: int, ldx: int, y_dev: int, ldy: int, stream: int = 0):
        check(bound_lib().lumina_gemv(self.handle, x_dev, int(batch), int(ldx), y_dev, int(ldy), stream))

    def gemm_rows(self, x_dev: int, rows: int, ldx: int, y_dev: int, ldy: int, stream: int = 0):
        """y = x W^T for many rows (prefill / verification) on tcgen05; int4
        weights in the tensor-core fragment layout."""
        check(bound_lib().lumina_gemm_rows(self.handle, x_dev, int(rows), int(ldx), y_dev, int(ldy), stream))

    def gemv_noalloc(self, x_dev: int, batch: int, ldx: int, y_dev: int, ldy: int, stream: int = 0):
        """``gemv`` without any device allocation: the activation scratch is
        the library's fixed 1 MiB device array (for callers that cannot
        allocate; calls that overlap on the GPU race on that array)."""
        check(bound_lib().lumina_gemv_noalloc(self.handle, x_dev, int(batch), int(ldx), y_dev, int(ldy), stream))

    def gemv_host(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
        assert x.shape[1] == self.cols
        y = np.empty((x.shape[0], self.rows), dtype=np.float32)
        check(bound_lib().lumina_gemv_host(self.handle, ptr(x, ctypes.c_float), x.shape[0],
                                           ptr(y, ctypes.c_float)))
        return y

    def __del__(self):
        try:
            if self._owned and self.handle:
                bound_lib().lumina_weight_free(self.handle)
                self.handle = None
        except Exception:  # noqa: BLE001
            pass


# ---------------------------------------------------------------------------
# tops-compatible int8 family (tops.py:296-420): {"out"} / {"error"}
# ---------------------------------------------------------------------------
def _guard(fn):
    def wrap(*a, **k):
        try:
            lib = ensure_device(0)
        except Exception as e:  # noqa: BLE001
            return {"error": str(e)}
        try:
            return fn(lib, *a, **k)
        except Exception as e:  # noqa: BLE001
            return {"error": str(e)}
    wrap.__name__ = fn.__name__
    wrap.__doc__ = fn.__doc__
    return wrap


@_guard
def gemv_int8(lib, xq, xs, wq, ws, out=None):
    """out[n] = ws[n] * sum_b dot(xq_block, wq_row_block) * xs[b] (tops.py:296-314)."""
    N, K = int(wq.shape[0]), int(wq.shape[1])
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    wq = np.ascontiguousarray(wq, dtype=np.int8)
    xs = np.ascontiguousarray(xs, dtype=np.float32)
    ws = np.ascontiguousarray(ws, dtype=np.float32).reshape(-1)
    if xq.shape[0] < K:
        return {"error": "xq shorter than K (pad to a 32-block first)"}
    o = np.zeros(N, dtype=np.float32)
    check(lib.lumina_gemv_int8(ptr(xq, ctypes.c_int8), ptr(xs, ctypes.c_float), ptr(wq, ctypes.c_int8),
                               ptr(ws, ctypes.c_float), ptr(o, ctypes.c_float), N, K), lib)
    if out is not None:
        out[...] = o
        o = out
    return {"out": o}


@_guard
def gemv_q4_0(lib, xq, xs, wq, ws, out=None):
    """Q4_0 GEMV: wq packed (N, K//2) uint8, ws (N, K//32) (tops.py:317-334)."""
    K, N = int(wq.shape[1]) * 2, int(wq.shape[0])
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    wq = np.ascontiguousarray(wq, dtype=np.uint8)
    xs = np.ascontiguousarray(xs, dtype=np.float32)
    ws = np.ascontiguousarray(ws, dtype=np.float32)
    o = np.zeros(N, dtype=np.float32)
    check(lib.lumina_gemv_q4_0(ptr(xq, ctypes.c_int8), ptr(xs, ctypes.c_float), ptr(wq, ctypes.c_uint8),
                               ptr(ws, ctypes.c_float), ptr(o, ctypes.c_float), N, K), lib)
    if out is not None:
        out[...] = o
        o = out
    return {"out": o}


@_guard
def gemv_fp16(lib, x, w, out=None):
    """fp16 GEMV with fp32 output (tops.py:390-400)."""
    N, K = int(w.shape[0]), int(w.shape[1])
    x = np.ascontiguousarray(x, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.float16)
    o = np.zeros(N, dtype=np.float32)
    check(lib.lumina_gemv_fp16(x.ctypes.data, w.ctypes.data, ptr(o, ctypes.c_float), N, K), lib)
    if out is not None:
        out[...] = o
        o = out
    return {"out": o}


@_guard
def gemm_int8(lib, xq, xs, wq, ws, out=None):
    """out[m,n] = ws[n] * sum_b dot(xq[m]_block, wq[n]_block) * xs[m,b] (tops.py:403-420)."""
    M, K = int(xq.shape[0]), int(xq.shape[1])
    N = int(wq.shape[0])
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    wq = np.ascontiguousarray(wq, dtype=np.int8)
    xs = np.ascontiguousarray(xs, dtype=np.float32)
    ws = np.ascontiguousarray(ws, dtype=np.float32).reshape(-1)
    o = np.zeros((M, N), dtype=np.float32)
    check(lib.lumina_gemm_int8(ptr(xq, ctypes.c_int8), ptr(xs, ctypes.c_float), ptr(wq, ctypes.c_int8),
                               ptr(ws, ctypes.c_float), ptr(o, ctypes.c_float), M, N, K), lib)
    if out is not None:
        out[...] = o
        o = out
    return {"out": o}
