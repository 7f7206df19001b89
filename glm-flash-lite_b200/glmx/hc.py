"""Drop-in for the reference's fused hyper-connection site extension (glm53/k_hcfuse.py: `ext().apply_partials` and
`ext().finalize_norm`, 296-344; used by `_site`, 427-432): the same function names, arguments and in-place outputs,
over libglmx's kernels (glmx_hc_apply_partials, glmx_hc_finalize_norm), bit-identical to the reference's kernels.

The MoE layer can run the first of them itself, in its combine: MoELayer.forward_hc(..., fn=, partials=).
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check


def _stream_ptr(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def check_mix_args(x: torch.Tensor, fn: torch.Tensor, partials: torch.Tensor) -> None:
    """x fp32 [R, 4, D] contiguous, fn fp16 [24, 4D] contiguous, partials fp32 with room for [R, 4D/128, 25]."""
    if x.dim() != 3 or x.shape[1] != 4 or x.dtype != torch.float32 or not x.is_contiguous() or x.shape[2] % 128:
        raise ValueError("x must be contiguous fp32 [R, 4, D] with D % 128 == 0")
    R, _, D = x.shape
    if fn is None or fn.dtype != torch.float16 or tuple(fn.shape) != (24, 4 * D) or not fn.is_contiguous():
        raise ValueError("fn must be contiguous fp16 (24, 4D)")
    if partials is None or partials.dtype != torch.float32 or not partials.is_contiguous() or \
            partials.numel() < R * (4 * D // 128) * 25:
        raise ValueError("partials must be contiguous fp32 with room for (R, 4D/128, 25)")
    for t in (x, fn, partials):
        if t.device != x.device:
            raise ValueError("x, fn and partials must be on one device")


def apply_partials(x: torch.Tensor, y: torch.Tensor | None, post: torch.Tensor | None, comb: torch.Tensor | None,
                   fn: torch.Tensor, partials: torch.Tensor, stream=None) -> None:
    """The reference's apply_partials (glm53/k_hcfuse.py:296-320): with y (fp16 or fp32 [R, D]) hc_apply of the
    pending site on x fp32 [R, 4, D] in place (post fp32 [R, 4], comb fp32 [R, 4, 4]); then the next site's
    hc_mix_partials of x into partials [R, 4D/128, 25]."""
    check_mix_args(x, fn, partials)
    R, _, D = x.shape
    yp = 0
    ydt = _lib.F32
    if y is not None:
        if y.dtype not in (torch.float16, torch.float32) or y.numel() != R * D or not y.is_contiguous():
            raise ValueError("y must be contiguous fp16/fp32 [R, D]")
        if post is None or comb is None:
            raise ValueError("y needs post and comb")
        post = post.to(torch.float32).contiguous(); comb = comb.to(torch.float32).contiguous()
        if post.numel() != R * 4 or comb.numel() != R * 16:
            raise ValueError("post must be [R, 4] and comb [R, 4, 4]")
        yp, ydt = y.data_ptr(), (_lib.F16 if y.dtype == torch.float16 else _lib.F32)
    L = _lib.load()
    check(L.glmx_hc_apply_partials(x.data_ptr(), yp, ydt, post.data_ptr() if y is not None else 0,
                                   comb.data_ptr() if y is not None else 0, fn.data_ptr(), partials.data_ptr(), R, D,
                                   _stream_ptr(stream)))


def finalize_norm(x: torch.Tensor, partials: torch.Tensor, base: torch.Tensor, scale: torch.Tensor, post: torch.Tensor,
                  comb: torch.Tensor, nw: torch.Tensor, out: torch.Tensor, rms_eps: float, hc_eps: float, iters: int,
                  n_eps: float, cbias: float, cscale: float, stream=None) -> None:
    """The reference's finalize_norm (glm53/k_hcfuse.py:322-344): hc_mix_finalize from the partials (post [R, 4],
    Sinkhorn comb [R, 4, 4]) and the site's RMSNorm of the collapsed row into out fp16 [R, D]; nw fp16 or bf16 [D]."""
    if x.dim() != 3 or x.shape[1] != 4 or x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("x must be contiguous fp32 [R, 4, D]")
    R, _, D = x.shape
    f32 = lambda t, n, what: _req(t, torch.float32, n, what)
    f32(partials, R * (4 * D // 128) * 25, "partials")
    f32(base, 24, "base"); f32(scale, 3, "scale"); f32(post, R * 4, "post"); f32(comb, R * 16, "comb")
    if nw.dtype not in (torch.float16, torch.bfloat16) or nw.numel() != D or not nw.is_contiguous():
        raise ValueError("nw must be contiguous fp16/bf16 [D]")
    _req(out, torch.float16, R * D, "out")
    L = _lib.load()
    check(L.glmx_hc_finalize_norm(x.data_ptr(), partials.data_ptr(), R, D, base.data_ptr(), scale.data_ptr(),
                                  post.data_ptr(), comb.data_ptr(), nw.data_ptr(),
                                  _lib.BF16 if nw.dtype == torch.bfloat16 else _lib.F16, out.data_ptr(), float(rms_eps),
                                  float(hc_eps), int(iters), float(n_eps), float(cbias), float(cscale),
                                  _stream_ptr(stream)))


def _req(t: torch.Tensor, dtype, n: int, what: str) -> None:
    if t.dtype != dtype or not t.is_contiguous() or t.numel() < n:
        raise ValueError(f"{what} must be contiguous {dtype} with {n} elements")
