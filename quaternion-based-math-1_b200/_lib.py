"""ctypes binding of the in-tree C ABI (``lib/libqlin_b200.so``).

This is the only way the package reaches the device: there is no CPU path and
no fallback.  A missing or unloadable library raises ``RuntimeError`` at the
first call.  Status codes from ``include/qlin_b200.h`` become exceptions with
the reference's classes: shape errors are ``ValueError``
(``quaternion/packing.py:45-52``), everything else ``RuntimeError``
(``kernels/cuda/quaternion_linear.cu:120-128,153``).
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libqlin_b200.so")

F32, BF16, F16 = 0, 1, 2
ALGO_AUTO, ALGO_SIMT, ALGO_TC, ALGO_GEMV = 0, 1, 2, 3
FLAG_STATIC_WEIGHTS = 1
FLAG_ZEROED_WORKSPACE = 2
FLAG_NO_PAIR = 4
FLAG_NO_CLUSTER = 8
PLAN_TC_PAIR = 4

OK = 0
ERR_SHAPE = 1
ERR_TIMEOUT = 7

_DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_lib = None
_fast = None  # CPython binding of qlin_forward_ex (lib/_qlin_call*.so), when built
_torch_ext = None  # C++ inference forward of the modules (lib/_qlin_torch*.so), when built
_lock = threading.Lock()

EXPORTED = (
    "qlin_status_string",
    "qlin_abi_version",
    "qlin_workspace_size",
    "qlin_forward",
    "qlin_forward_ex",
    "qlin_select_algo",
    "qlin_plan",
    "qlin_get_device_error",
    "qlin_gather_columns",
    "qlin_forward_noalloc",
    "qlin_forward_packed",
    "qlin_forward_allgather",
    "qlin_forward_allgather_mc",
    "qlin_ipc_alloc",
    "qlin_ipc_free",
    "qlin_ipc_open",
    "qlin_ipc_close",
    "qlin_forward_host",
    "qlin_host_workspace_size",
    "qlin_sharded_fwd",
    "qlin_sharded_workspace_size",
    "qlin_nccl_unique_id",
    "qlin_nccl_comm_init",
    "qlin_nccl_comm_destroy",
)


def load(path: str | None = None):
    """Load (once) and return the ctypes handle of the C ABI library."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"quaternion linear CUDA library not built ({p}); run "
                "`python quaternion-based-math-1_b200/build.py` (nvcc, sm_100a)"
            )
        lib = ctypes.CDLL(p)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        lib.qlin_status_string.argtypes = [I]
        lib.qlin_status_string.restype = ctypes.c_char_p
        lib.qlin_abi_version.restype = I
        lib.qlin_workspace_size.argtypes = [I, I64, I64, I64, I, ctypes.POINTER(ctypes.c_size_t)]
        lib.qlin_workspace_size.restype = I
        fwd = [I, P, I64, P, P, P, P, I64, P, P, P, I, ctypes.c_float, P, I64, I64, I64, I64,
               P, ctypes.c_size_t]
        lib.qlin_forward.argtypes = fwd + [P]
        lib.qlin_forward.restype = I
        lib.qlin_forward_ex.argtypes = fwd + [I, I, P]
        lib.qlin_forward_ex.restype = I
        lib.qlin_select_algo.argtypes = [I, I64, I64, I64, I]
        lib.qlin_select_algo.restype = I
        IP = ctypes.POINTER(I)
        lib.qlin_plan.argtypes = [I, I64, I64, I64, I, I, IP, IP, IP, IP, IP]
        lib.qlin_plan.restype = I
        lib.qlin_get_device_error.argtypes = [P, I, ctypes.POINTER(I)]
        lib.qlin_get_device_error.restype = I
        lib.qlin_forward_packed.argtypes = ([I, P, I64, P, I64, P, P, P, P, I64, P, P, P, I, ctypes.c_float, P, I64,
                                             I64, I64, I64, P, ctypes.c_size_t, I, P])
        lib.qlin_forward_packed.restype = I
        lib.qlin_forward_noalloc.argtypes = fwd[:-2] + [P]
        lib.qlin_forward_noalloc.restype = I
        lib.qlin_gather_columns.argtypes = [I, P, P, I64, I64, I64, I64, P]
        lib.qlin_gather_columns.restype = I
        PP = ctypes.POINTER(P)
        lib.qlin_forward_allgather.argtypes = (
            [I, P, I64, P, P, P, P, I64, P, P, P, I, ctypes.c_float, I64, I64, I64, P, ctypes.c_size_t, I,
             I, I, PP, I64, I64, PP, P, P])
        lib.qlin_forward_allgather.restype = I
        lib.qlin_forward_allgather_mc.argtypes = (
            [I, P, I64, P, P, P, P, I64, P, P, P, I, ctypes.c_float, I64, I64, I64, P, ctypes.c_size_t, I,
             I, I, P, P, I64, I64, PP, P, P])
        lib.qlin_forward_allgather_mc.restype = I
        lib.qlin_ipc_alloc.argtypes = [ctypes.c_size_t, PP, ctypes.c_char_p]
        lib.qlin_ipc_alloc.restype = I
        lib.qlin_ipc_free.argtypes = [P]
        lib.qlin_ipc_free.restype = I
        lib.qlin_ipc_open.argtypes = [ctypes.c_char_p, I64, PP]
        lib.qlin_ipc_open.restype = I
        lib.qlin_ipc_close.argtypes = [P]
        lib.qlin_ipc_close.restype = I
        lib.qlin_sharded_fwd.argtypes = [I, P, I64, P, P, P, P, I64, P, P, P, I, ctypes.c_float, P, I64, I64, I64,
                                         I64, P, ctypes.c_size_t, I, P, I, I, P]
        lib.qlin_sharded_fwd.restype = I
        lib.qlin_forward_host.argtypes = fwd + [I, I, P]
        lib.qlin_forward_host.restype = I
        lib.qlin_host_workspace_size.argtypes = [I, I64, I64, I64, I, ctypes.POINTER(ctypes.c_size_t)]
        lib.qlin_host_workspace_size.restype = I
        lib.qlin_sharded_workspace_size.argtypes = [I, I64, I64, I64, I, I, ctypes.POINTER(ctypes.c_size_t)]
        lib.qlin_sharded_workspace_size.restype = I
        lib.qlin_nccl_unique_id.argtypes = [ctypes.c_char_p]
        lib.qlin_nccl_unique_id.restype = I
        lib.qlin_nccl_comm_init.argtypes = [PP, I, ctypes.c_char_p, I]
        lib.qlin_nccl_comm_init.restype = I
        lib.qlin_nccl_comm_destroy.argtypes = [P]
        lib.qlin_nccl_comm_destroy.restype = I
        if path is None:
            _lib = lib
            _load_fast(os.path.dirname(p))
        return lib


def _load_fast(lib_dir: str) -> None:
    """Import the bindings built next to the library (both link to the same
    libqlin_b200.so, already loaded above): the CPython binding of
    qlin_forward_ex and the C++ inference forward; keep ctypes and the Python
    forward without them."""
    global _fast, _torch_ext
    import glob
    import importlib.util

    def imp(pattern, name):
        for f in glob.glob(os.path.join(lib_dir, pattern)):
            spec = importlib.util.spec_from_file_location(name, f)
            if spec is None or spec.loader is None:
                continue
            try:
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
            except ImportError:
                continue
            return mod
        return None

    _fast = imp("_qlin_call*.so", "_qlin_call")
    _torch_ext = imp("_qlin_torch*.so", "_qlin_torch")


def status_string(code: int) -> str:
    return load().qlin_status_string(int(code)).decode()


def check(code: int, what: str) -> None:
    if code == OK:
        return
    msg = f"{what}: {status_string(code)} (status {code})"
    if code == ERR_SHAPE:
        raise ValueError(msg)
    raise RuntimeError(msg)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise RuntimeError(
            f"unsupported dtype {dtype}; the B200 quaternion kernels take float32, bfloat16 "
            "or float16"
        ) from None


def stream_handle(device: torch.device) -> int:
    """Raw handle of the current CUDA stream of ``device`` (cudaStream_t as int)."""
    return torch._C._cuda_getCurrentRawStream(device.index if device.index is not None
                                              else torch.cuda.current_device())


_ws_sizes: dict[tuple, int] = {}


def workspace_size(dtype: torch.dtype, M: int, K_g: int, N_g: int, rank: int) -> int:
    key = (dtype, M, K_g, N_g, rank)
    n = _ws_sizes.get(key)
    if n is None:
        c = ctypes.c_size_t(0)
        check(load().qlin_workspace_size(dtype_code(dtype), M, K_g, N_g, rank, ctypes.byref(c)),
              "qlin_workspace_size")
        n = _ws_sizes[key] = int(c.value)
    return n


def device_error(device: torch.device | None = None, clear: bool = True) -> int:
    """Synchronise the current stream and return (and clear) the device error word."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    st = ctypes.c_int(0)
    with torch.cuda.device(dev):
        check(load().qlin_get_device_error(stream_handle(dev), int(clear), ctypes.byref(st)),
              "qlin_get_device_error")
    return int(st.value)


def plan(dtype: torch.dtype, M: int, K_g: int, N_g: int, rank: int, flags: int | None = None) -> dict:
    """Launch plan on the current device (see qlin_plan).  ``flags`` defaults
    to the flags :func:`forward_raw` passes for this problem."""
    if flags is None:
        flags = FLAG_ZEROED_WORKSPACE if _uses_zeroed_workspace(dtype, M) else 0
    outs = [ctypes.c_int(0) for _ in range(5)]
    check(load().qlin_plan(dtype_code(dtype), M, K_g, N_g, rank, int(flags),
                           *(ctypes.byref(o) for o in outs)),
          "qlin_plan")
    algo, tok, split, launches, resident = (o.value for o in outs)
    return {"algo": {ALGO_SIMT: "simt", ALGO_TC: "tcgen05", ALGO_GEMV: "gemv",
                     PLAN_TC_PAIR: "tcgen05-pair"}.get(algo, str(algo)),
            "tile_tokens": tok, "split_k": split, "launches": launches, "resident_ctas": resident}


def _ptr(t):
    return None if t is None else t.data_ptr()


# Decode-sized calls (few tokens) run on a zero-filled workspace kept per
# (device, stream): with QLIN_FLAG_ZEROED_WORKSPACE their K split is summed
# inside the main kernel, one launch fewer.  Calls on one stream are ordered,
# so they may share it; each call leaves its counter bytes at zero.
_ZEROED_MAX_TOKENS = 4
_zeroed_ws: dict[tuple[int, int], torch.Tensor] = {}
# Buffers replaced by larger ones are never released: a CUDA graph captured
# earlier on the same stream still holds their addresses.
_zeroed_retired: list[torch.Tensor] = []


def _uses_zeroed_workspace(dtype: torch.dtype, M: int) -> bool:
    return dtype in (torch.bfloat16, torch.float16) and 0 < M <= _ZEROED_MAX_TOKENS


def zeroed_workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """The zero-filled workspace of the current stream of ``device``, grown to
    ``nbytes`` if needed; None while a CUDA graph is being captured and the
    cached buffer is too small (the caller then uses a plain workspace)."""
    key = (device.index, stream_handle(device))
    buf = _zeroed_ws.get(key)
    if buf is not None and buf.numel() >= nbytes:
        return buf
    if torch.cuda.is_current_stream_capturing():
        return None
    if buf is not None:
        _zeroed_retired.append(buf)
    buf = torch.zeros(max(nbytes, 64 * 1024), dtype=torch.uint8, device=device)
    _zeroed_ws[key] = buf
    return buf


def forward_raw(x2, ld_x, w, ld_w, bias, lora_a, lora_b, rank, lora_scale, y2, ld_y,
                M, K_g, N_g, algo=ALGO_AUTO, flags=0, packed=None):
    """Call ``qlin_forward_ex`` (``qlin_forward_packed`` with a packed weight
    cache and the automatic kernel choice) on prepared 2-D device tensors
    (see linear.py)."""
    lib = _lib if _lib is not None else load()
    dev = x2.device
    ws_bytes = workspace_size(x2.dtype, M, K_g, N_g, rank)
    ws = None
    if ws_bytes and _uses_zeroed_workspace(x2.dtype, M):
        ws = zeroed_workspace(dev, ws_bytes)
        if ws is not None:
            flags |= FLAG_ZEROED_WORKSPACE
    if ws is None and ws_bytes:
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    if packed is not None and algo == ALGO_AUTO:
        code = lib.qlin_forward_packed(
            _DTYPE_CODE[x2.dtype], x2.data_ptr(), ld_x, packed.data_ptr(), K_g, w[0].data_ptr(), w[1].data_ptr(),
            w[2].data_ptr(), w[3].data_ptr(), ld_w, _ptr(bias), _ptr(lora_a), _ptr(lora_b), rank, lora_scale,
            y2.data_ptr(), ld_y, M, K_g, N_g, _ptr(ws), ws_bytes, flags,
            torch._C._cuda_getCurrentRawStream(dev.index))
        check(code, "qlin_forward_packed")
        return y2
    fn = _fast.forward_ex if _fast is not None else lib.qlin_forward_ex
    code = fn(
        _DTYPE_CODE[x2.dtype], x2.data_ptr(), ld_x, w[0].data_ptr(), w[1].data_ptr(), w[2].data_ptr(),
        w[3].data_ptr(), ld_w, _ptr(bias), _ptr(lora_a), _ptr(lora_b), rank, lora_scale,
        y2.data_ptr(), ld_y, M, K_g, N_g, _ptr(ws), ws_bytes, algo, flags,
        torch._C._cuda_getCurrentRawStream(dev.index),
    )
    check(code, "qlin_forward")
    return y2
