"""ctypes binding of libqmoe_b200.so (the C ABI declared in include/qmoe_b200.h).

The library is the only compute path: if it is missing, or the current CUDA device is not an
sm_100 part, every call raises. There is no CPU or PyTorch fallback.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqmoe_b200.so")

OK = 0
DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_c = ctypes
_p = _c.c_void_p
_i = _c.c_int
_i64 = _c.c_int64
_f = _c.c_float
_sz = _c.c_size_t

# name -> (restype, argtypes); one entry per function of include/qmoe_b200.h
SIGNATURES = {
    "qmoe_version": (_c.c_char_p, []),
    "qmoe_status_string": (_c.c_char_p, [_i]),
    "qmoe_workspace_status": (_i, [_p, _i, _p]),
    "qmoe_decode_up": (_i, [_p, _i64, _i64, _p, _i, _p, _p, _i, _p, _p]),
    "qmoe_live_groups": (_i, [_p, _i, _p, _p, _p]),
    "qmoe_decode_down_groups": (_i, [_p, _p, _p, _p, _p, _p, _i, _i, _p, _p]),
    "qmoe_decode_groups_workspace_bytes": (_sz, [_i]),
    "qmoe_decode_groups": (_i, [_p, _i64, _i64, _p, _p, _p, _p, _p, _i, _i, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "qmoe_decode_groups_static": (_i, [_p, _i64, _i64, _p, _p, _p, _p, _p, _i, _i, _p, _p, _p, _p, _p, _p]),
    "qmoe_decode_groups_static_status": (_i, [_i, _p]),
    "qmoe_decode": (_i, [_p, _i64, _i64, _p, _p, _p, _p, _i, _i, _p, _p, _p, _p]),
    "qmoe_pairs": (_i, [_p, _i64, _i64, _p, _p, _p, _p, _p, _i, _i, _i, _p, _p, _p]),
    "qmoe_set_wait_cycles": (_i, [_c.c_longlong]),
    "qmoe_copy_async": (_i, [_p, _p, _sz, _p]),
    "dq_gemv_bf16": (_i, [_p, _p, _i, _i, _i, _i, _i, _p, _p, _p]),
    "dq_gemv_nvfp4_bf16": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _p, _p, _p]),
    "qmoe_route_decode": (_i, [_p, _p, _i, _i, _c.c_float, _i, _p, _i64, _p, _p, _p, _p, _p, _p, _p]),
    "qmoe_prefill_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "qmoe_prefill_grouped": (_i, [_p, _i64, _i, _i, _p, _p, _p, _p, _i, _i, _i, _p, _p, _sz, _p]),
    "qmoe_ep_dispatch_pack": (_i, [_p, _i, _p, _p, _i, _i, _i, _i, _p, _p, _p, _p, _p]),
    "qmoe_ep_combine": (_i, [_p, _p, _i, _i, _p, _p]),
    "qmoe_from_T": (_i, [_p, _i, _p, _p]),
    "qmoe_to_T": (_i, [_p, _i, _p, _p]),
    "qmoe_deq": (_i, [_p, _p, _f, _i64, _i64, _p, _p]),
    "qmoe_block_deq": (_i, [_p, _f, _f, _p, _p, _p]),
    "dq_gemv_fp8": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p]),
    "dq_gemv_nvfp4": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _p, _p]),
    "dq_dequant_rows": (_i, [_i, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i, _p]),
}

_lib = None


class QmoeError(RuntimeError):
    pass


def lib():
    """Load the library (once). Raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise QmoeError(f"{LIB_PATH} is missing: build it with qmoe_build.py (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def status_string(code):
    return lib().qmoe_status_string(int(code)).decode()


def check(code, name):
    if code != OK:
        raise QmoeError(f"{name}: {status_string(code)} (status {code})")


def call(name, *args):
    check(getattr(lib(), name)(*args), name)


def stream_of(t=None):
    """cudaStream_t of torch's current stream on the tensor's device."""
    dev = t.device if t is not None else None
    return torch.cuda.current_stream(dev).cuda_stream


def ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise QmoeError("libqmoe_b200 works on CUDA tensors only (got a CPU tensor)")
    return t.data_ptr()


def dtype_code(t):
    try:
        return DT[t.dtype]
    except KeyError:
        raise QmoeError(f"unsupported activation dtype {t.dtype}") from None


def version():
    return lib().qmoe_version().decode()
