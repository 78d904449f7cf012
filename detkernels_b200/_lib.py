"""ctypes binding of the detkernels_b200 C ABI (include/detkernels_b200.h).

Loads the in-tree ``libdetkernels_b200.so``.  There is no fallback: if the
library is missing every op raises, on any machine.  Torch is used only for
device memory, the current stream and tensor metadata.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

# ---- status / dtype codes (mirror include/detkernels_b200.h) ----
DK_OK = 0
DK_ERR_INVALID_ARGUMENT = 1
DK_ERR_UNSUPPORTED = 2
DK_ERR_WORKSPACE = 3
DK_ERR_CUDA = 4
DK_ERR_DEVICE_TIMEOUT = 5
DK_ERR_DEVICE_CHECK = 6

DK_F32 = 0
DK_F16 = 1
DK_BF16 = 2

MATMUL_K_SLICES = 8
ATTN_KV_SPLIT = 256

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_int = ctypes.c_int
_f32 = ctypes.c_float
_size = ctypes.c_size_t

# name -> (restype, argtypes); every symbol declared in include/detkernels_b200.h
SIGNATURES = {
    "dk_abi_version": (_int, []),
    "dk_last_error": (ctypes.c_char_p, []),
    "dk_device_status": (_int, [_int, _int, ctypes.POINTER(_int), ctypes.POINTER(_int)]),
    "dk_num_sms": (_int, [_int, ctypes.POINTER(_int)]),
    "dk_test_bounded_wait": (_int, [_int, _i64, _c_void_p]),
    "dk_kernel_attributes": (_int, [_int, ctypes.POINTER(_int), ctypes.POINTER(_int), ctypes.POINTER(_int),
                                    ctypes.POINTER(_int)]),
    "dk_rmsnorm_batch_invariant": (_int, [_c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64, _int, _int,
                                          _f32, _c_void_p]),
    "dk_rmsnorm_gather_batch_invariant": (_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64,
                                                 _c_void_p, _i64, _i64, _i64, _int, _int, _f32, _c_void_p]),
    "dk_rmsnorm_variant_workspace_size": (_size, [_i64]),
    "dk_rmsnorm_batch_variant": (_int, [_c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64, _int, _int, _f32,
                                        _int, _int, _c_void_p, _size, _c_void_p]),
    "dk_matmul_workspace_size": (_size, [_i64, _i64, _i64]),
    "dk_matmul_batch_invariant": (_int, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _i64, _i64, _i64, _int,
                                         _c_void_p, _size, _c_void_p]),
    "dk_matmul_batch_invariant_ex": (_int, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _i64, _i64, _i64,
                                            _int, _c_void_p, _c_void_p, _size, _c_void_p]),
    "dk_gdn_forward": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64,
                              _int, _int, _int, _int, _int, _int, ctypes.c_float, _c_void_p, _int, _c_void_p, _int,
                              _c_void_p]),
    "dk_argmax_finish": (_int, [_c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "dk_matmul_fold_slices_ex": (_int, [_c_void_p, _int, _c_void_p, _i64, _i64, _i64, _int, _c_void_p, _c_void_p]),
    "dk_argmax_finish_parts": (_int, [_c_void_p, _int, _i64, ctypes.POINTER(_i64), _i64, _c_void_p, _c_void_p,
                                      _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "dk_matmul_shard_range": (None, [_i64, _int, _int, _c_void_p, _c_void_p]),
    "dk_matmul_shard_partials": (_int, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _i64, _i64, _int, _int,
                                        _int, _c_void_p]),
    "dk_matmul_slice_partials": (_int, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _i64, _i64, _int, _int,
                                        _int, _c_void_p]),
    "dk_matmul_fold_slices": (_int, [_c_void_p, _int, _c_void_p, _i64, _i64, _i64, _int, _c_void_p]),
    "dk_matmul_variant_workspace_size": (_size, [_i64, _i64]),
    "dk_matmul_batch_variant": (_int, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _i64, _i64, _i64, _int,
                                       _int, _int, _c_void_p, _size, _c_void_p]),
    "dk_attention_workspace_size": (_size, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "dk_attention_batch_invariant": (_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64,
                                            _i64, _c_void_p, _i64, _i64, _c_void_p, _i32, _c_void_p, _i32, _i32,
                                            _i32, _i32, _i32, _i32, _f32, _int, _c_void_p, _size, _c_void_p]),
    "dk_attention_paged_batch_invariant": (_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64,
                                                  _i64, _i32, _c_void_p, _i64, _i64, _i32, _c_void_p, _i64, _i64,
                                                  _c_void_p, _i32, _c_void_p, _i32, _i32, _i32, _i32, _i32, _i32,
                                                  _f32, _int, _c_void_p, _size, _c_void_p]),
    "dk_attention_noalloc_scratch_limit": (_size, []),
    "dk_attention_batch_invariant_noalloc": (_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64,
                                                    _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i32, _c_void_p,
                                                    _i32, _i32, _i32, _i32, _i32, _i32, _f32, _int, _c_void_p]),
    "dk_attention_variant_workspace_size": (_size, [_i32, _i32, _i32]),
    "dk_attention_batch_variant": (_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p,
                                          _i64, _i64, _i32, _i32, _i32, _i32, _f32, _i32, _int, _c_void_p, _size,
                                          _c_void_p]),
}


# layout version of the structs mirrored here (DK_ABI_VERSION of include/detkernels_b200.h)
ABI_VERSION = 3

DK_EPI_STORE = 0
DK_EPI_RESIDUAL = 1
DK_EPI_SILU = 2
DK_EPI_SILU_MUL = 3
DK_EPI_QKV_CACHE = 4
DK_EPI_ARGMAX = 5
DK_EPI_RESIDUAL_RMSNORM = 6


class MatmulEpilogue(ctypes.Structure):
    """ctypes mirror of dk_matmul_epilogue."""
    _fields_ = [("mode", ctypes.c_int), ("resid", ctypes.c_void_p), ("ld_resid", ctypes.c_int64),
                ("q_cols", ctypes.c_int32), ("kv_cols", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
                ("cache_stride_seq", ctypes.c_int64), ("cache_stride_head", ctypes.c_int64),
                ("cache_stride_tok", ctypes.c_int64), ("row_seq", ctypes.c_void_p), ("row_pos", ctypes.c_void_p),
                ("argmax_keys", ctypes.c_void_p), ("norm_w", ctypes.c_void_p), ("norm_w_dtype", ctypes.c_int),
                ("norm_out", ctypes.c_void_p), ("norm_ld", ctypes.c_int64), ("norm_eps", ctypes.c_float),
                ("block_table", ctypes.c_void_p), ("block_table_stride", ctypes.c_int64),
                ("page_size", ctypes.c_int32), ("blocks_per_seq", ctypes.c_int32), ("n_blocks", ctypes.c_int64)]


class DetKernelsError(RuntimeError):
    """A non-zero status from the C ABI or from the device status word."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lock = threading.Lock()
_lib = None


def library_path() -> str:
    return _build.LIB_PATH


def load():
    """Load the in-tree library (it is never built here: ``python -m detkernels_b200.build``
    or ``__graft_entry__.build()`` builds it).  A missing library, a library of another ABI
    version or one that lacks a declared entry point raises DetKernelsError."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        rebuild = "rebuild it with `python -m detkernels_b200.build`"
        if not os.path.exists(path):
            raise DetKernelsError(
                DK_ERR_CUDA,
                "detkernels_b200: %s is not built; run `python -m detkernels_b200.build` "
                "(there is no CPU or eager fallback)" % path)
        lib = ctypes.CDLL(path)
        try:
            version_fn = lib.dk_abi_version
        except AttributeError:
            raise DetKernelsError(DK_ERR_UNSUPPORTED, "detkernels_b200: %s exports no dk_abi_version; %s"
                                  % (path, rebuild)) from None
        version_fn.restype = _int
        version_fn.argtypes = []
        if version_fn() != ABI_VERSION:
            raise DetKernelsError(
                DK_ERR_UNSUPPORTED,
                "detkernels_b200: %s has ABI version %d, this package needs %d; %s"
                % (path, version_fn(), ABI_VERSION, rebuild))
        for name, (res, args) in SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError:
                raise DetKernelsError(DK_ERR_UNSUPPORTED, "detkernels_b200: %s lacks %s (a stale build); %s"
                                      % (path, name, rebuild)) from None
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().dk_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc == DK_OK:
        return
    msg = "%s failed (code %d): %s" % (what, rc, last_error())
    if rc == DK_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == DK_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise DetKernelsError(rc, msg)


def device_status(device: int, clear: bool = True):
    """(code, detail) of the device status word; synchronises the device."""
    code = _int(0)
    detail = _int(0)
    check(load().dk_device_status(int(device), 1 if clear else 0, ctypes.byref(code), ctypes.byref(detail)),
          "dk_device_status")
    return code.value, detail.value


def raise_on_device_error(device: int) -> None:
    code, detail = device_status(device, clear=True)
    if code != DK_OK:
        if code in (DK_ERR_DEVICE_TIMEOUT, DK_ERR_DEVICE_CHECK):
            # scratch counters may be mid-update; start from clean workspaces
            reset_workspaces(device)
        raise DetKernelsError(code, "device status %d (detail 0x%x) on cuda:%d" % (code, detail, device))


# ---- launch accounting (host side): every wrapper that launches one of this
# library's kernels adds to it; captured CUDA graphs record the count at capture ----
_launches = [0]


def count_launch(n: int = 1) -> None:
    _launches[0] += n


def launch_count() -> int:
    return _launches[0]


# ---- torch glue ----
def dtype_code(dtype) -> int:
    import torch
    if dtype == torch.float32:
        return DK_F32
    if dtype == torch.float16:
        return DK_F16
    if dtype == torch.bfloat16:
        return DK_BF16
    raise NotImplementedError("detkernels_b200: unsupported dtype %s" % (dtype,))


def stream_ptr(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


_workspaces = {}
_ws_lock = threading.Lock()


def workspace(nbytes: int, device, stream: int):
    """Zero-initialised scratch buffer of >= nbytes for (device, stream).

    Arrival counters inside the scratch reset themselves at the end of every
    launch, so a buffer is reused as is.  Calls that overlap on different
    streams get different buffers."""
    import torch
    if nbytes <= 0:
        return None
    dev = torch.device(device)
    key = (dev.index, stream)
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(int(nbytes), 1 << 20)
            if buf is not None:
                size = max(size, 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=dev)
            _workspaces[key] = buf
        return buf


def reset_workspaces(device=None) -> None:
    with _ws_lock:
        for key in list(_workspaces):
            if device is None or key[0] == device:
                _workspaces[key].zero_()


def exported_symbols():
    return list(SIGNATURES)


def kernel_attributes(which: int):
    """(registers/thread, max threads/block, local bytes, max dynamic smem) of a compiled kernel."""
    vals = [_int(0) for _ in range(4)]
    check(load().dk_kernel_attributes(int(which), *[ctypes.byref(v) for v in vals]), "dk_kernel_attributes")
    return tuple(v.value for v in vals)
