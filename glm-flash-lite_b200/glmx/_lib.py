"""ctypes binding of libglmx.so (the C ABI in include/glmx.h). Fails loudly when the library is missing: there is
no CPU fallback for any entry point."""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.environ.get("GLMX_LIB") or os.path.join(PKG, "lib", "libglmx.so")   # GLMX_LIB: another build of it

F16, F32, BF16, I32, I64 = 0, 1, 2, 3, 4
MODE_EXACT = 1
MODE_I16 = 2
PATH_GEMV, PATH_GEMM = 0x100, 0x200    # OR'ed into MODE_EXACT: force the decode GEMV or the prefill GEMM kernels
PHASES = 6
OK, E_ARG, E_CUDA, E_DEVICE, E_WORKSPACE = 0, -1, -2, -3, -4
ABI_VERSION = 2

_P = C.c_void_p
_I = C.c_int


class LayerDesc(C.Structure):
    """glmx_layer_desc of include/glmx.h"""
    _fields_ = [("hidden", _I), ("intermediate", _I), ("n_experts", _I), ("has_shared", _I),
                ("bits", _I * 3), ("trellis", _P), ("suh", _P * 3), ("svh", _P * 3), ("act_limit", C.c_float),
                ("first_expert", _I)]


class PeerOut(C.Structure):
    """glmx_peer_out of include/glmx.h"""
    _fields_ = [("recv", _P), ("flags", _P), ("counter", _P), ("rank", _I), ("world", _I), ("rows_per_rank", _I),
                ("seq", _I)]


class GlmxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"glmx error {code}: {msg}")
        self.code = code


# every symbol include/glmx.h declares
EXPORTS = ("glmx_version", "glmx_last_error", "glmx_layer_create", "glmx_layer_destroy", "glmx_layer_set_act_limit",
           "glmx_workspace_bytes", "glmx_route", "glmx_workspace_array", "glmx_moe_forward", "glmx_moe_forward_timed",
           "glmx_decode_tiles", "glmx_check", "glmx_moe_forward_noalloc", "glmx_moe_forward_hc",
           "glmx_moe_forward_hc_mix", "glmx_hc_apply_partials", "glmx_hc_finalize_norm",
           "glmx_selftest_bounded_wait", "glmx_router", "glmx_moe_forward_peer", "glmx_peer_reduce", "glmx_ep_split", "glmx_ipc_alloc",
           "glmx_ipc_free", "glmx_ipc_handle", "glmx_ipc_open", "glmx_ipc_close", "glmx_layer_device", "glmx_check_noalloc",
           "glmx_ep_pack", "glmx_ep_unpack_add")
IPC_HANDLE_BYTES = 64
NOALLOC_SCRATCH_BYTES = 48 << 20
ROUTER_MAX_EXPERTS = 512

_lib = None


def load(path: str = LIB_PATH):
    """Load libglmx.so once. Raises FileNotFoundError if it was not built (glm-flash-lite_b200/build.sh)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} missing: build it with glm-flash-lite_b200/build.sh (there is no CPU fallback)")
    L = C.CDLL(path)
    L.glmx_version.restype = _I
    L.glmx_last_error.restype = C.c_char_p
    L.glmx_layer_create.argtypes = [C.POINTER(LayerDesc), C.POINTER(_P)]
    L.glmx_layer_create.restype = _I
    L.glmx_layer_destroy.argtypes = [_P]
    L.glmx_layer_destroy.restype = _I
    L.glmx_layer_set_act_limit.argtypes = [_P, C.c_float]
    L.glmx_layer_set_act_limit.restype = _I
    L.glmx_workspace_bytes.argtypes = [_P, _I, _I]
    L.glmx_workspace_bytes.restype = C.c_size_t
    L.glmx_route.argtypes = [_P, _P, _I, _P, _I, _I, _I, _P, C.c_size_t, _P]
    L.glmx_route.restype = _I
    L.glmx_workspace_array.argtypes = [_P, _I, _I, _I, C.POINTER(C.c_size_t)]
    L.glmx_workspace_array.restype = _I
    L.glmx_moe_forward.argtypes = [_P, _P, _I, _I, _P, _I, _P, _I, _I, _I, _P, _I, _I, _P, C.c_size_t, _P]
    L.glmx_moe_forward.restype = _I
    L.glmx_moe_forward_timed.argtypes = [_P, _P, _I, _I, _P, _I, _P, _I, _I, _I, _P, _I, _I, _P, C.c_size_t, _P, _P]
    L.glmx_moe_forward_timed.restype = _I
    L.glmx_decode_tiles.argtypes = [_P, _I, _I, _P, _P]
    L.glmx_decode_tiles.restype = _I
    L.glmx_check.argtypes = [_P, _I, _I, _P, _P, C.POINTER(_I)]
    L.glmx_check.restype = _I
    L.glmx_moe_forward_noalloc.argtypes = [_P, _P, _I, _I, _P, _I, _P, _I, _I, _I, _P, _I, _I, _P]
    L.glmx_moe_forward_noalloc.restype = _I
    L.glmx_ep_pack.argtypes = [_P, _P, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P, _P, _P, _P]
    L.glmx_ep_pack.restype = _I
    L.glmx_ep_unpack_add.argtypes = [_P, _P, _I, _I, _I, _P, _P]
    L.glmx_ep_unpack_add.restype = _I
    L.glmx_check_noalloc.argtypes = [_P, _I, _I, _P, C.POINTER(_I)]
    L.glmx_check_noalloc.restype = _I
    L.glmx_layer_device.argtypes = [_P]
    L.glmx_layer_device.restype = _I
    L.glmx_moe_forward_hc.argtypes = [_P, _P, _I, _I, _P, _I, _P, _I, _I, _I, _P, _P, _P, _I, _P, C.c_size_t, _P]
    L.glmx_moe_forward_hc.restype = _I
    L.glmx_moe_forward_hc_mix.argtypes = [_P, _P, _I, _I, _P, _I, _P, _I, _I, _I, _P, _P, _P, _I, _P, _P, _P, C.c_size_t,
                                          _P]
    L.glmx_moe_forward_hc_mix.restype = _I
    L.glmx_hc_apply_partials.argtypes = [_P, _P, _I, _P, _P, _P, _P, _I, _I, _P]
    L.glmx_hc_apply_partials.restype = _I
    L.glmx_hc_finalize_norm.argtypes = [_P, _P, _I, _I, _P, _P, _P, _P, _P, _I, _P, C.c_float, C.c_float, _I, C.c_float,
                                        C.c_float, C.c_float, _P]
    L.glmx_hc_finalize_norm.restype = _I
    L.glmx_selftest_bounded_wait.argtypes = [_I, _P, _P]
    L.glmx_selftest_bounded_wait.restype = _I
    L.glmx_router.argtypes = [_P, _I, _I, _I, _P, _I, _P, _I, _I, _I, _I, _I, C.c_float, _P, _P, _I, _P, _I, _P]
    L.glmx_router.restype = _I
    L.glmx_moe_forward_peer.argtypes = [_P, _P, _I, _I, _P, _I, _P, _I, _I, _I, C.POINTER(PeerOut), _P, C.c_size_t, _P]
    L.glmx_moe_forward_peer.restype = _I
    L.glmx_peer_reduce.argtypes = [_P, _P, _I, _I, _I, _I, _P, _I, _P, _P]
    L.glmx_peer_reduce.restype = _I
    L.glmx_ep_split.argtypes = [_P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P]
    L.glmx_ep_split.restype = _I
    L.glmx_ipc_alloc.argtypes = [C.c_size_t, C.POINTER(_P)]
    L.glmx_ipc_alloc.restype = _I
    L.glmx_ipc_free.argtypes = [_P]
    L.glmx_ipc_free.restype = _I
    L.glmx_ipc_handle.argtypes = [_P, _P]
    L.glmx_ipc_handle.restype = _I
    L.glmx_ipc_open.argtypes = [_P, C.POINTER(_P)]
    L.glmx_ipc_open.restype = _I
    L.glmx_ipc_close.argtypes = [_P]
    L.glmx_ipc_close.restype = _I
    if L.glmx_version() != ABI_VERSION:
        raise RuntimeError(f"libglmx ABI {L.glmx_version()} != {ABI_VERSION}")
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != OK:
        raise GlmxError(rc, (load().glmx_last_error() or b"").decode())
