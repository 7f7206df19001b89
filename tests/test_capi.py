"""The C-ABI library loads and exports every entry point include/glmx.h declares (no compute calls: CPU only)."""
import ctypes as C
import os
import re

from conftest import REPO


def declared_symbols():
    src = open(os.path.join(REPO, "include", "glmx.h")).read()
    return sorted(set(re.findall(r"GLMX_API\s+[\w\s\*]+?\b(glmx_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "glmx_moe_forward" in names and "glmx_route" in names and "glmx_decode_tiles" in names


def test_library_exports_every_declared_symbol():
    from glmx import _lib
    L = _lib.load()
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert set(_lib.EXPORTS) == set(declared_symbols())


def test_version_and_error_without_gpu():
    from glmx import _lib
    L = _lib.load()
    assert L.glmx_version() == _lib.ABI_VERSION
    # argument validation happens before any CUDA call
    rc = L.glmx_layer_create(None, None)
    assert rc == _lib.E_ARG
    assert b"null" in L.glmx_last_error()
    d = _lib.LayerDesc()
    d.hidden, d.intermediate, d.n_experts = 100, 256, 4
    h = C.c_void_p()
    assert L.glmx_layer_create(C.byref(d), C.byref(h)) == _lib.E_ARG
    assert b"multiples of 128" in L.glmx_last_error()
    assert L.glmx_decode_tiles(None, 5, 1, None, None) == _lib.E_ARG
    assert L.glmx_selftest_bounded_wait(0, None, None) == _lib.E_ARG
    assert b"timeout_us" in L.glmx_last_error()
    R = lambda E, ng, tg, k, ntok=4: L.glmx_router(None, _lib.F32, ntok, 0, None, _lib.F32, None, E, ng, tg, k, 1, 1.0,
                                                   None, None, _lib.I32, None, _lib.F32, None)
    assert R(513, 1, 1, 8) == _lib.E_ARG                  # more experts than the selection scratch holds
    assert R(288, 5, 1, 8) == _lib.E_ARG                  # groups must divide the experts
    assert R(288, 8, 2, 80) == _lib.E_ARG                 # topk beyond the kept groups
    assert R(288, 1, 1, 8) == _lib.E_ARG and b"required" in L.glmx_last_error()   # null outputs
    assert R(288, 1, 1, 8, ntok=-1) == _lib.E_ARG
    assert L.glmx_peer_reduce(None, None, 2, 4, 256, 1, None, _lib.F32, None, None) == _lib.E_ARG
    assert L.glmx_ep_split(None, 4, 0, 0, 36, 1, 0, 4, None, None, None) == _lib.E_ARG       # topk 0
    assert L.glmx_ep_split(None, 0, 8, 0, 36, 1, 0, 0, None, None, None) == _lib.OK          # nothing to do
    assert L.glmx_moe_forward_peer(None, None, _lib.F16, 2, None, _lib.I32, None, _lib.F32, 8, 2, None, None, 0, None) == _lib.E_ARG
