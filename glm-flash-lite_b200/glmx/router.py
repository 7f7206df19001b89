"""Router of the MoE site on the GPU (glmx_router): gate linear, sigmoid, score-correction bias, group-limited top-k,
renormalised weights — the GLM-4 MoE routing that exllamav3's router hands to the reference's routing_fn hook
(glm53/cpu_tier.py:305-335), as transformers states it (models/glm4_moe/modeling_glm4_moe.py:302-305, 389-412).
Its (sel, w) feed MoELayer.forward directly on the device."""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check
from .layer import _dt, _stream_ptr


class Router:
    """weight: [E, H] gate matrix (fp32, bf16 or fp16 CUDA tensor) or None (then __call__ takes logits);
    bias: e_score_correction_bias fp32 [E] or None; the rest as the published config names them
    (num_experts_per_tok, n_group, topk_group, norm_topk_prob, routed_scaling_factor)."""

    def __init__(self, weight=None, bias=None, topk: int = 8, n_group: int = 1, topk_group: int = 1,
                 norm: bool = True, scale: float = 1.0, n_experts: int | None = None):
        self.lib = _lib.load()
        self.weight = None if weight is None else weight.contiguous()
        self.E = int(self.weight.shape[0]) if self.weight is not None else int(n_experts)
        self.bias = None if bias is None else bias.to(torch.float32).contiguous()
        self.topk, self.n_group, self.topk_group = int(topk), int(n_group), int(topk_group)
        self.norm, self.scale = bool(norm), float(scale)

    def _run(self, z, logits, ntok, sel_dtype, w_dtype, stream):
        dev = logits.device
        sel = torch.empty((ntok, self.topk), dtype=sel_dtype, device=dev)
        w = torch.empty((ntok, self.topk), dtype=w_dtype, device=dev)
        check(self.lib.glmx_router(
            None if z is None else z.data_ptr(), _lib.F32 if z is None else _dt(z), ntok,
            0 if z is None else int(z.shape[-1]),
            None if self.weight is None else self.weight.data_ptr(), _lib.F32 if self.weight is None else _dt(self.weight),
            None if self.bias is None else self.bias.data_ptr(), self.E, self.n_group, self.topk_group, self.topk,
            int(self.norm), self.scale, logits.data_ptr(), sel.data_ptr(), _dt(sel), w.data_ptr(), _dt(w),
            _stream_ptr(stream)))
        return sel, w

    def __call__(self, z: torch.Tensor, sel_dtype=torch.int32, w_dtype=torch.float32, stream=None):
        """z [ntok, H] -> (sel [ntok, topk], w [ntok, topk], logits fp32 [ntok, E])."""
        if self.weight is None:
            raise ValueError("this Router has no gate weight: use select(logits)")
        z = z.reshape(-1, z.shape[-1]).contiguous()
        logits = torch.empty((z.shape[0], self.E), dtype=torch.float32, device=z.device)
        sel, w = self._run(z, logits, z.shape[0], sel_dtype, w_dtype, stream)
        return sel, w, logits

    def select(self, logits: torch.Tensor, sel_dtype=torch.int32, w_dtype=torch.float32, stream=None):
        """fp32 logits [ntok, E] -> (sel, w)."""
        logits = logits.to(torch.float32).contiguous()
        return self._run(None, logits, logits.shape[0], sel_dtype, w_dtype, stream)
