"""Test infrastructure: builds the reference's own fused hyper-connection kernels (glm53/k_hcfuse.py, the CUDA source
string `_SRC` with its `apply_partials` / `finalize_norm` host functions) into oracle/_ref/hc/glm53_k101.so, as the
reference builds them (torch extension, nvcc -O3 --use_fast_math, k_hcfuse.py:355-365), for sm_100a.

The source is read from the reference tree beside the repository (REF_ROOT overrides) and compiled where it lies in the
build folder oracle/_ref/hc (git-ignored; the built module travels with the repository snapshot to the GPU box, where
tests/golden/make_hc_golden.py runs it to write the hc golden fixtures). Nothing of it is committed.
"""
from __future__ import annotations

import ast
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "hc")
SO = os.path.join(OUT, "glm53_k101.so")
REF_ROOT_DEFAULT = os.path.normpath(os.path.join(HERE, "..", "..", "reference"))


def reference_source(ref_root: str) -> str:
    """The `_SRC` string constant of glm53/k_hcfuse.py (read as text, not imported)."""
    path = os.path.join(ref_root, "glm53", "k_hcfuse.py")
    tree = ast.parse(open(path).read(), path)
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == "_SRC" for t in node.targets):
            return node.value.value
    raise RuntimeError(f"no _SRC in {path}")


def build(ref_root: str | None = None) -> str | None:
    """Build the module; returns its path, or None when the reference tree is absent."""
    ref_root = ref_root or os.environ.get("REF_ROOT", REF_ROOT_DEFAULT)
    if not os.path.isfile(os.path.join(ref_root, "glm53", "k_hcfuse.py")):
        return None
    src = reference_source(ref_root)
    os.makedirs(OUT, exist_ok=True)
    cu = os.path.join(OUT, "k101.cu")
    if not os.path.exists(cu) or open(cu).read() != src:
        open(cu, "w").write(src)
    if os.path.exists(SO) and os.path.getmtime(SO) >= os.path.getmtime(cu):
        return SO
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load
    load(name="glm53_k101", sources=[cu], build_directory=OUT,
         extra_cuda_cflags=["-lineinfo", "-O3", "--use_fast_math"], verbose=False)
    return SO


def load_built():
    """Import the prebuilt module from oracle/_ref/hc (no reference tree needed)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the module links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader("glm53_k101", SO)
    spec = importlib.util.spec_from_file_location("glm53_k101", SO, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None))
