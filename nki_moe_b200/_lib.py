"""ctypes binding of ``libnkimoe.so`` (the C ABI in ``include/nkimoe.h``).

There is no fallback: if the library is missing or fails to load, every
operation raises.  Error codes from the C ABI become ``NKIMoEError`` (a
``RuntimeError``) carrying the code and the library's message, the same
surface a reference user gets from a failing kernel call.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("NKIMOE_LIB", os.path.join(_HERE, "libnkimoe.so"))

OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_DEVICE = 5

F32, BF16, I32, I64 = 0, 1, 2, 3
LAYOUT_NXD, LAYOUT_HF = 0, 1

_c = ctypes
_vp, _i, _i64, _f, _sz = _c.c_void_p, _c.c_int, _c.c_int64, _c.c_float, _c.c_size_t

# name -> (restype, argtypes); the list is the C ABI this package binds.
SIGNATURES = {
    "nkimoe_version": (_i, []),
    "nkimoe_last_error": (_c.c_char_p, []),
    "nkimoe_set_option": (_i, [_c.c_char_p, _c.c_longlong]),
    "nkimoe_set_stage_events": (_i, [_c.POINTER(_vp), _i]),
    "nkimoe_rmsnorm": (_i, [_vp, _i, _vp, _i, _vp, _i, _i64, _i64, _f, _vp]),
    "nkimoe_add_rmsnorm": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _i64, _i64, _f, _vp]),
    "nkimoe_qk_norm_rope": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _i64, _i, _i, _i, _f, _f, _vp]),
    "nkimoe_decode_attention_workspace_bytes": (_sz, [_i64, _i, _i, _i, _i64]),
    "nkimoe_decode_attention": (_i, [_vp, _vp, _vp, _i, _vp, _i64, _vp, _vp, _vp, _i64, _i, _i, _i, _i64, _f, _f, _f,
                                     _vp, _sz, _vp]),
    "nkimoe_skinny_linear": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "nkimoe_router_logits": (_i, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "nkimoe_topk_softmax": (_i, [_vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "nkimoe_permute_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "nkimoe_permute": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "nkimoe_pack_gate_up": (_i, [_vp, _i, _vp, _i64, _i64, _i64, _vp]),
    "nkimoe_pack_down": (_i, [_vp, _i, _vp, _i64, _i64, _i64, _vp]),
    "nkimoe_moe_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "nkimoe_moe_experts": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _vp]),
    "nkimoe_moe_block": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _sz,
                              _vp]),
    "nkimoe_moe_block_add_rmsnorm": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _f, _vp, _vp, _vp, _i64,
                                          _i64, _i64, _i64, _i64, _vp, _sz, _vp]),
    "nkimoe_moe_block_rmsnorm_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "nkimoe_moe_block_rmsnorm": (_i, [_vp, _vp, _i, _f, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                      _i64, _i64, _vp, _sz, _vp]),
    "nkimoe_moe_block_host_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "nkimoe_moe_block_host_plan": (_i, [_i64, _i64, _i64, _i, _i64, _vp, _vp]),
    "nkimoe_moe_block_host": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                   _vp, _sz, _vp, _vp]),
    "nkimoe_router_split": (_i, [_vp, _vp, _i64, _i64, _vp]),
    "nkimoe_read_status": (_i, [_vp, _vp, _c.POINTER(_i)]),
    "nkimoe_noalloc_read_status": (_i, [_vp, _c.POINTER(_i)]),
    "nkimoe_moe_block_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                      _vp]),
    "nkimoe_grouped_gemm": (_i, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "nkimoe_route_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "nkimoe_route": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _sz, _vp]),
    "nkimoe_dispatch_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "nkimoe_dispatch": (_i, [_vp, _vp, _i, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "nkimoe_segment_experts_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "nkimoe_segment_experts": (_i, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "nkimoe_combine": (_i, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "nkimoe_ep_peer_buffer_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "nkimoe_peer_alloc": (_i, [_sz, _c.POINTER(_vp), _vp]),
    "nkimoe_peer_open": (_i, [_vp, _c.POINTER(_vp)]),
    "nkimoe_peer_close": (_i, [_vp]),
    "nkimoe_peer_free": (_i, [_vp]),
    "nkimoe_ep_peer_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _i64]),
    "nkimoe_ep_peer_schedule": (_i, [_i64, _i64]),
    "nkimoe_ep_peer_forward": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                    _i64, _i64, _c.POINTER(_vp), _c.c_uint32, _vp, _sz, _vp]),
    "nkimoe_ep_peer_workspace_bytes_mapped": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64]),
    "nkimoe_ep_peer_forward_mapped": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                           _i64, _i64, _i64, _c.POINTER(_vp), _c.c_uint32, _vp, _sz, _vp, _i64, _vp,
                                           _vp, _i64]),
    "nkimoe_ep_dispatch_workspace_bytes": (_sz, [_i64, _i64]),
    "nkimoe_ep_dispatch": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                                _vp]),
    "nkimoe_swiglu": (_i, [_vp, _vp, _i64, _i64, _vp]),
    "nkimoe_aggregate": (_i, [_vp, _vp, _i64, _i64, _i64, _vp]),
}


class NKIMoEError(RuntimeError):
    def __init__(self, code: int, fn: str, msg: str):
        super().__init__(f"{fn} failed with code {code}: {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the CUDA library (once).  Raises if it is absent: there is no
    CPU or PyTorch fallback for any operation of this package."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"libnkimoe.so not found at {LIB_PATH}; build it with `python -m nki_moe_b200.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name: str, *args) -> int:
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        msg = lib.nkimoe_last_error().decode(errors="replace")
        raise NKIMoEError(rc, name, msg)
    return rc


def size_call(name: str, *args) -> int:
    return int(getattr(load(), name)(*args))


def set_option(name: str, value: int) -> None:
    call("nkimoe_set_option", name.encode(), int(value))
