"""ctypes binding of libsoupsuck_b200.so (the C ABI declared in include/soupsuck_b200.h).

The product path has no fallback: if the shared library is missing or a CUDA
device is unavailable, every kernel entry raises.  Argument validation that the
reference performs in Python (ValueError before any launch) happens in the
``kernels`` modules; a non-zero status from the library raises ValueError for
SB_EINVAL and RuntimeError otherwise, with the library's message.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libsoupsuck_b200.so"

SB_OK, SB_EINVAL, SB_ECUDA, SB_EUNSUPPORTED, SB_EWORKSPACE = 0, 1, 2, 3, 4
SB_F16, SB_F32 = 0, 1

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_F32 = ctypes.c_float
_SZ = ctypes.c_size_t
_PI64 = ctypes.POINTER(ctypes.c_int64)


class NF4Weight(ctypes.Structure):
    _fields_ = [("packed", _P), ("qabs", _P), ("absmax2", _P), ("code2", _P), ("offset", _P),
                ("n_out", _I64), ("k_in", _I64)]


# name -> (restype, argtypes); mirrors include/soupsuck_b200.h
SIGNATURES = {
    "sb_abi_version": (_I32, []),
    "sb_last_error": (ctypes.c_char_p, []),
    "sb_take_device_error": (_I32, [_P, ctypes.POINTER(_I32)]),
    "sb_launch_count": (_I64, []),
    "sb_nf4_dequant_nested": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _P]),
    "sb_nf4_dequant_flat": (_I32, [_P, _P, _P, _I64, _P]),
    "sb_nf4_linear_fwd": (_I32, [_P, _I64, ctypes.POINTER(NF4Weight), _P, _P, _P, _I32, _P, _P, _SZ, _P]),
    "sb_nf4_linear_dx": (_I32, [_P, _I64, ctypes.POINTER(NF4Weight), _P, _P, _I32, _P, _P, _SZ, _P]),
    "sb_nf4_linear_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32]),
    "sb_lora_prepare": (_I32, [_P, _I32, _P, _I32, _I32, _I64, _I64, _P, _P, _P, _P, _P]),
    "sb_lora_prepare_pair": (_I32, [_P, _P, _I32, _P, _P, _I32, _I32, _I64, _I64, _P, _P, _P, _P, _P]),
    "sb_lora_project": (_I32, [_P, _I64, _I64, _P, _I32, _F32, _P, _I32, _F32, _P, _I64, _P]),
    "sb_lora_reduce_workspace_bytes": (_SZ, [_I64, _I64, _I32]),
    "sb_lora_reduce": (_I32, [_P, _I64, _P, _I64, _I64, _I32, _F32, _I32, _P, _I32, _P, _SZ, _P]),
    "sb_lora_dual_workspace_bytes": (_SZ, [_I64, _I64, _I32, _I64]),
    "sb_lora_dual": (_I32, [_P, _I64, _I64, _P, _I64, _P, _I32, _I64, _F32, _I32, _P, _I32,
                            _F32, _P, _I32, _F32, _P, _I64, _P, _SZ, _P]),
    "sb_lora_reduce_static": (_I32, [_P, _I64, _P, _I64, _I64, _I32, _F32, _I32, _P, _I32, _P]),
    "sb_lora_scale_add": (_I32, [_P, _I32, _P, _I32, _P, _I32, _I64, _F32, _I32, _P]),
    "sb_lora_scale_grad": (_I32, [_P, _I32, _P, _I32, _I64, _F32, _P]),
    "sb_add_rmsnorm_fwd": (_I32, [_P, _I32, _P, _I32, _P, _I32, _I64, _P, _P, _I32, _P, _I64, _I64, _F32, _P]),
    "sb_add_rmsnorm_bwd": (_I32, [_P, _I32, _P, _I32, _I64, _P, _P, _I32, _I64, _I64, _P, _I32, _I64,
                                  _I64, _P, _I32, _P, _I32, _I64, _I64, _P]),
    "sb_rmsnorm_fwd": (_I32, [_P, _I32, _I64, _P, _I32, _I64, _P, _I32, _P, _I64, _I64, _F32, _P]),
    "sb_rmsnorm_input_grad": (_I32, [_P, _I32, _I64, _P, _I32, _I64, _P, _I32, _I64, _I64, _P, _P,
                                     _I64, _I64, _P]),
    "sb_rmsnorm_weight_grad": (_I32, [_P, _I32, _I64, _P, _I32, _I64, _I64, _P, _P, _I32, _I64, _I64,
                                      _I32, _P, _SZ, _P]),
    "sb_rmsnorm_weight_grad_workspace_bytes": (_SZ, [_I64, _I64]),
    "sb_ce_forward": (_I32, [_P, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _SZ, _P]),
    "sb_ce_forward_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sb_ce_forward_shard": (_I32, [_P, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "sb_ce_backward": (_I32, [_P, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I32, _P, _SZ, _P]),
    "sb_ce_backward_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sb_ce_check_targets": (_I32, [_P, _I64, _I64, _I64, ctypes.POINTER(_I64), _P]),
    "sb_rope": (_I32, [_P, _I32, _PI64, _I64, _P, _I32, _P, _I32, _PI64, _I64, _P, _I32, _P, _P, _I32,
                       _PI64, _PI64, _I64, _I64, _I64, _I64, _I32, _P]),
    "sb_swiglu_fwd": (_I32, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _P]),
    "sb_swiglu_bwd": (_I32, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _P]),
    "sb_nf4_mlp_gate_up_fwd": (_I32, [_P, _I64, ctypes.POINTER(NF4Weight), ctypes.POINTER(NF4Weight), _P, _P,
                                      _I32, _P, _P, _P]),
    "sb_nf4_mlp_down_dx": (_I32, [_P, _I64, ctypes.POINTER(NF4Weight), _P, _P, _I32, _P, _P, _P]),
    "sb_nf4_linear_dx2_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sb_nf4_linear_dx2": (_I32, [_P, _I64, ctypes.POINTER(NF4Weight), ctypes.POINTER(NF4Weight), _P, _P, _I32,
                                 _P, _P, _SZ, _P]),
    "sb_unpad_workspace_bytes": (_SZ, [_I64]),
    "sb_unpad_metadata": (_I32, [_P, _I32, _P, _I64, _I64, _I64, _P, _P, _SZ, _P]),
    "sb_unpad_pack": (_I32, [_P, _I64, _I64, _I64, _P, _I64, _P, _P]),
    "sb_unpad_scatter": (_I32, [_P, _I64, _I64, _I64, _P, _P, _P]),
}

_lock = threading.Lock()
_lib = None


def load():
    """Load the shared library once; raise RuntimeError if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m soupsuck_b200.build` "
                    "(there is no CPU or Python fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name, *args):
    """Invoke an entry point and turn a non-zero status into an exception."""
    rc = getattr(load(), name)(*args)
    if rc != SB_OK:
        msg = load().sb_last_error().decode(errors="replace")
        if rc == SB_EINVAL:
            raise ValueError(f"{name}: {msg}")
        raise RuntimeError(f"{name} failed ({rc}): {msg}")
    return rc


def query(name, *args) -> int:
    return int(getattr(load(), name)(*args))


def stream_of(device) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype) -> int:
    import torch
    if dtype == torch.float16:
        return SB_F16
    if dtype == torch.float32:
        return SB_F32
    raise ValueError(f"unsupported dtype {dtype}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def launch_count() -> int:
    return int(load().sb_launch_count())


def take_device_error(device=None) -> int:
    flag = _I32(0)
    call("sb_take_device_error", stream_of(device), ctypes.byref(flag))
    return int(flag.value)
