"""ctypes binding of the C ABI in ``include/memintelli_b200.h``.

The library is the only compute path: there is no CPU or PyTorch fallback.
``lib()`` raises when the shared object has not been built.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

c_i32, c_i64, c_u64, c_f32, c_f64, c_vp = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float,
                                           ctypes.c_double, ctypes.c_void_p)

MIB_OK = 0
MIB_ERR_PARAM = 1
MIB_ERR_SHAPE = 2
MIB_ERR_UNSUPPORTED = 3
MIB_ERR_CUDA = 4
MIB_ERR_TIMEOUT = 5

OPERAND_E4M3 = 0
OPERAND_FP16 = 1
OPERAND_FP16_SPLIT = 2     # FP16 inputs; weights as FP16 hi planes followed by FP16 lo planes

MODE_LUT = 1
MODE_FLOATACC = 2


class SliceSpec(ctypes.Structure):
    _fields_ = [("n_slices", c_i32), ("slice_method", c_i32 * 8), ("bfp", c_i32), ("paral", c_i32 * 2),
                ("quant_gran", c_i32 * 2)]


class DeviceSpec(ctypes.Structure):
    _fields_ = [("hgs", c_f64), ("lgs", c_f64), ("g_level", c_i32), ("rdac", c_i32), ("n_radc", c_i32),
                ("radc", c_i32 * 8), ("vread", c_f64), ("vnoise", c_f64), ("write_variation", c_f64),
                ("rate_stuck_hgs", c_f64), ("rate_stuck_lgs", c_f64), ("n_read_sigma", c_i32),
                ("read_sigma", c_f32 * 256)]


class OutLayout(ctypes.Structure):
    _fields_ = [("rows_per_group", c_i64), ("group_stride", c_i64), ("row_stride", c_i64), ("col_stride", c_i64)]


class KGeom(ctypes.Structure):
    _fields_ = [("k", c_i64), ("kp", c_i64), ("p", c_i32), ("pp", c_i32), ("kt", c_i64)]


_P = ctypes.POINTER
_SIGS = {
    "mib_slice_input": [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, _P(SliceSpec), _P(KGeom), c_i32, c_i32,
                        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    "mib_slice_rmsnorm_input": [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_f32, _P(SliceSpec),
                                _P(KGeom), c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    "mib_slice_swiglu_input": [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, _P(SliceSpec), _P(KGeom), c_i32,
                               c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    "mib_qk_norm_rope_bf16": [c_vp, c_i64, c_i64, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_f32, c_vp, c_vp, c_vp,
                              c_vp, c_vp, c_vp],
    "mib_slice_conv_input": [c_vp, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                             _P(SliceSpec), _P(KGeom), c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    "mib_slice_conv_input_noisy": [c_vp, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                                   c_i32, _P(SliceSpec), _P(KGeom), c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_f64, c_u64,
                                   c_u64, c_vp],
    "mib_program_weight": [c_vp, c_i64, c_i64, c_i64, c_i64, _P(SliceSpec), _P(KGeom), _P(DeviceSpec), c_vp, c_vp,
                           c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    "mib_input_noise": [c_vp, c_vp, c_i64, c_f64, c_u64, c_u64, c_vp],
    "mib_weight_read_noise": [c_vp, c_vp, c_vp, c_i64, _P(DeviceSpec), c_u64, c_u64, c_vp],
    "mib_weight_read_noise_split": [c_vp, c_vp, c_vp, c_i64, _P(DeviceSpec), c_u64, c_u64, c_vp],
    "mib_weight_read_noise_background": [c_vp, c_vp, c_vp, c_i64, _P(DeviceSpec), c_u64, c_u64, c_i32, c_i32, c_vp],
    "mib_adc_plan": [_P(SliceSpec), _P(SliceSpec), _P(KGeom), _P(DeviceSpec), _P(c_i32), _P(c_i32), c_vp],
    "mib_mvm": [c_vp, c_vp, c_i64, _P(SliceSpec), c_vp, c_vp, c_i64, _P(SliceSpec), _P(KGeom), _P(DeviceSpec), c_i32,
                c_vp, c_i32, c_vp, _P(OutLayout), c_vp, c_vp, c_vp, c_i64, c_vp],
    "mib_mvm_workspace": [c_i64, c_i64, _P(SliceSpec), _P(SliceSpec), _P(KGeom), _P(DeviceSpec), _P(c_i64)],
    "mib_mvm_static_scratch": [c_vp, c_vp, c_i64, _P(SliceSpec), c_vp, c_vp, c_i64, _P(SliceSpec), _P(KGeom),
                               _P(DeviceSpec), c_i32, c_vp, c_i32, c_vp, _P(OutLayout), c_vp, c_vp],
    "mib_row_logsumexp": [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp],
    "mib_device_status": [],
    "mib_test_inject_wait_expiry": [c_i64],
}
EXPORTS = tuple(_SIGS) + ("mib_last_error", "mib_version", "mib_launch_count")

_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    return _build.LIB


def lib():
    """Load the native library (once).  Raises RuntimeError if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(f"memintelli_flash_b200 native library not built ({path}); "
                                   "run `python -m memintelli_flash_b200.build`")
            L = ctypes.CDLL(path)
            for name, args in _SIGS.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = c_i32
            L.mib_last_error.restype = ctypes.c_char_p
            L.mib_last_error.argtypes = []
            L.mib_version.restype = ctypes.c_char_p
            L.mib_version.argtypes = []
            L.mib_launch_count.restype = ctypes.c_uint64
            L.mib_launch_count.argtypes = []
            _lib = L
    return _lib


_EXC = {MIB_ERR_PARAM: ValueError, MIB_ERR_SHAPE: ValueError, MIB_ERR_UNSUPPORTED: NotImplementedError,
        MIB_ERR_CUDA: RuntimeError, MIB_ERR_TIMEOUT: RuntimeError}


def check(rc: int):
    if rc != MIB_OK:
        msg = lib().mib_last_error().decode(errors="replace")
        raise _EXC.get(rc, RuntimeError)(msg)


def call(name: str, *args):
    check(getattr(lib(), name)(*args))


def ptr(t):
    """Device pointer of a tensor (or None)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device=None):
    """The current CUDA stream of ``device`` (a torch.device, an index or None for the current
    device) as a cudaStream_t.  Uses torch's raw-stream query when it is there: the public
    ``torch.cuda.current_stream`` costs several microseconds per call on the per-layer host path."""
    import torch
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        if device is None:
            idx = torch.cuda.current_device()
        elif isinstance(device, int):
            idx = device
        else:
            device = torch.device(device)
            idx = device.index if device.index is not None else torch.cuda.current_device()
        return ctypes.c_void_p(raw(idx))
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class _NoGuard:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


_NO_GUARD = _NoGuard()


def device_guard(device):
    """Context that makes ``device`` the current CUDA device for the native calls inside it.

    The library launches on the current device (and sets per-device kernel attributes there), so
    a call whose buffers live on another device must switch to it first.  Returns a no-op context
    when ``device`` is already current, which keeps the per-layer host path cheap."""
    import torch
    idx = device.index if isinstance(device, torch.device) else device
    if idx is None or idx == torch.cuda.current_device():
        return _NO_GUARD
    return torch.cuda.device(idx)


def launch_count() -> int:
    """Kernels launched by the native library so far in this process."""
    return int(lib().mib_launch_count())


def device_status():
    """Raise if a kernel on the current device gave up a bounded wait."""
    check(lib().mib_device_status())
