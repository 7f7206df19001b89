"""Host side of one routed-expert MoE layer: torch owns device memory and streams, libglmx does the work."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import check

_DT = {torch.float16: _lib.F16, torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.int32: _lib.I32,
       torch.int64: _lib.I64}

# which-array ids of glmx_workspace_array
WS_OFFSETS, WS_ROW_TOKEN, WS_ROW_WEIGHT, WS_PICK_ROW, WS_JOBS, WS_PLAN, WS_ROW_PICK = range(7)


def _stream_ptr(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


class MoELayer:
    """One MoE layer of E routed experts (+ optional shared expert) resident in HBM.

    trellis_ptrs: int64 [E_total, 3] device addresses of the native-layout gate / up / down trellis tensors (the pointer
    table exllamav3 keeps per expert, glm53/expert_cache.py:603-616, and tier_add_layer's `ptrs`, ft_tier_ext.cpp:160).
    suh / svh: three fp16 CUDA tensors each, [E_total, k] and [E_total, n] (tier_add_layer's scale shapes).
    keep: tensors that own the memory behind trellis_ptrs (kept alive by the layer).
    first_expert: global id of routed expert 0 (an expert-parallel shard); picks outside the shard are skipped.
    """

    def __init__(self, H: int, I: int, E: int, trellis_ptrs, suh, svh, bits=(3, 3, 3), has_shared: bool = False,
                 act_limit: float = 0.0, keep=(), device=None, first_expert: int = 0):
        self.lib = _lib.load()
        self.H, self.I, self.E = int(H), int(I), int(E)
        self.has_shared = bool(has_shared)
        self.bits = tuple(int(b) for b in bits)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.index is None:                    # "cuda" means the current device, as in torch
            self.device = torch.device("cuda", torch.cuda.current_device())
        et = self.E + (1 if self.has_shared else 0)
        ptrs = torch.as_tensor(trellis_ptrs, dtype=torch.int64).reshape(-1)
        if ptrs.numel() != et * 3:
            raise ValueError(f"trellis_ptrs must be [{et}, 3]")
        self.suh = [self._scale(s, et, k) for s, k in zip(suh, (self.H, self.H, self.I))]
        self.svh = [self._scale(s, et, n) for s, n in zip(svh, (self.I, self.I, self.H))]
        self._ptrs = np.ascontiguousarray(ptrs.cpu().numpy().astype(np.uint64))
        self.keep = list(keep)
        d = _lib.LayerDesc()
        d.hidden, d.intermediate, d.n_experts, d.has_shared = self.H, self.I, self.E, int(self.has_shared)
        for p in range(3):
            d.bits[p] = self.bits[p]
            d.suh[p] = self.suh[p].data_ptr()
            d.svh[p] = self.svh[p].data_ptr()
        d.trellis = self._ptrs.ctypes.data
        d.act_limit = float(act_limit)
        d.first_expert = int(first_expert)
        self.first_expert = int(first_expert)
        h = C.c_void_p()
        with torch.cuda.device(self.device):
            check(self.lib.glmx_layer_create(C.byref(d), C.byref(h)))
        self.h = h
        self._ws = None
        self.act_limit = float(act_limit)

    def _scale(self, s, et, dim):
        t = torch.as_tensor(s)
        if t.shape != (et, dim):
            raise ValueError(f"scale tensor must be [{et}, {dim}], got {tuple(t.shape)}")
        return t.to(device=self.device, dtype=torch.float16).contiguous()

    @classmethod
    def from_bank(cls, bank, device="cuda", act_limit: float = 0.0):
        """Upload a synth.ExpertBank (packed: per expert gate | up | down) into one HBM allocation."""
        dev = torch.device(device)
        tr = torch.from_numpy(bank.trellis).to(dev)
        base = tr.data_ptr()
        et = bank.e_total
        ptrs = np.array([[base + bank.proj_offset(e, p) for p in range(3)] for e in range(et)], dtype=np.int64)
        suh = [torch.from_numpy(s).to(dev) for s in bank.suh]
        svh = [torch.from_numpy(s).to(dev) for s in bank.svh]
        return cls(bank.H, bank.I, bank.E, ptrs, suh, svh, bits=bank.bits, has_shared=bank.shared,
                   act_limit=act_limit, keep=[tr], device=dev)

    def __del__(self):
        try:
            if getattr(self, "h", None) and self.h.value:
                self.lib.glmx_layer_destroy(self.h)
                self.h = C.c_void_p()
        except Exception:
            pass

    def set_act_limit(self, limit: float) -> None:
        check(self.lib.glmx_layer_set_act_limit(self.h, float(limit)))
        self.act_limit = float(limit)

    # ---- workspace --------------------------------------------------------------------------------------------
    def workspace_bytes(self, ntok: int, topk: int) -> int:
        return int(self.lib.glmx_workspace_bytes(self.h, int(ntok), int(topk)))

    def workspace(self, ntok: int, topk: int) -> torch.Tensor:
        need = self.workspace_bytes(ntok, topk)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=self.device)
        return self._ws

    def ws_array(self, ws: torch.Tensor, ntok: int, topk: int, which: int, dtype, count: int) -> torch.Tensor:
        off = C.c_size_t()
        check(self.lib.glmx_workspace_array(self.h, int(ntok), int(topk), int(which), C.byref(off)))
        item = torch.empty((), dtype=dtype).element_size()
        return ws[off.value:off.value + count * item].view(dtype)

    # ---- calls --------------------------------------------------------------------------------------------------
    def route(self, sel: torch.Tensor, w: torch.Tensor, stream=None) -> dict:
        """Top-k token split only; returns views of the routing arrays inside the workspace."""
        sel = sel.contiguous(); w = w.contiguous()
        ntok, topk = sel.shape
        ws = self.workspace(ntok, topk)
        check(self.lib.glmx_route(self.h, sel.data_ptr(), _dt(sel), w.data_ptr(), _dt(w), ntok, topk, ws.data_ptr(),
                                  ws.numel(), _stream_ptr(stream)))
        plan = self.ws_array(ws, ntok, topk, WS_PLAN, torch.int32, 8)
        return dict(ws=ws, plan=plan, ntok=ntok, topk=topk)

    def route_arrays(self, r: dict) -> dict:
        """Host copies of the routing arrays of a finished route() call (synchronises)."""
        ws, ntok, topk = r["ws"], r["ntok"], r["topk"]
        plan = r["plan"].cpu().numpy()
        P, R, J = int(plan[0]), int(plan[1]), int(plan[2])
        g = lambda which, dt, n: self.ws_array(ws, ntok, topk, which, dt, n).cpu().numpy()
        return dict(P=P, R=R, J=J, S_gu=int(plan[3]), S_d=int(plan[4]),
                    offsets=g(WS_OFFSETS, torch.int32, self.E + 1), row_token=g(WS_ROW_TOKEN, torch.int32, R),
                    row_weight=g(WS_ROW_WEIGHT, torch.float32, R), row_pick=g(WS_ROW_PICK, torch.int32, R),
                    pick_row=g(WS_PICK_ROW, torch.int32, ntok * topk),
                    jobs=g(WS_JOBS, torch.int32, 4 * J).reshape(J, 4))

    def forward(self, x: torch.Tensor, sel: torch.Tensor, w: torch.Tensor, mode: int = _lib.MODE_EXACT,
                out: torch.Tensor | None = None, out_dtype=torch.float32, accumulate: bool = False,
                stream=None, events=None, workspace: torch.Tensor | None = None) -> torch.Tensor:
        """out [ntok, H] = sum over each token's picks of w * expert(x) (+ shared expert).
        mode: 1 EXACT (default: fp16 codebook weights, fp32 accumulation, the reference's EXACT arithmetic), 2 I16
        (bit-identical to the reference's I16 kernel; int16 activations, outside the 2e-3 bar at H=6144).
        events: optional list of _lib.PHASES torch.cuda.Event recorded between the kernels on the launching stream.
        workspace: a uint8 CUDA tensor of at least workspace_bytes(ntok, topk) to use instead of the layer's own (calls
        that may run at the same time on different streams need workspaces of their own)."""
        x = x.contiguous(); sel = sel.contiguous(); w = w.contiguous()
        ntok = x.shape[0]
        topk = sel.shape[1] if sel.dim() == 2 else 0
        if x.shape[1] != self.H or sel.shape[0] != ntok or w.shape != sel.shape:
            raise ValueError("shape mismatch: x [ntok, H], sel/w [ntok, topk]")
        for t in (x, sel, w):
            if t.device != self.device:
                raise ValueError(f"tensor on {t.device}, layer on {self.device}")
        if out is None:
            out = torch.empty((ntok, self.H), dtype=out_dtype, device=self.device)
        if workspace is not None:
            if workspace.numel() < self.workspace_bytes(ntok, topk) or workspace.device != self.device:
                raise ValueError("workspace too small or on another device")
            ws = workspace
        else:
            ws = self.workspace(ntok, topk)
        ev = None
        if events is not None:
            for e in events:
                if e is not None and not e.cuda_event:
                    e.record(stream if stream is not None else torch.cuda.current_stream())   # creates the event
            ev = (C.c_void_p * _lib.PHASES)(*[e.cuda_event if e is not None else 0 for e in events])
        check(self.lib.glmx_moe_forward_timed(self.h, x.data_ptr(), _dt(x), ntok, sel.data_ptr(), _dt(sel), w.data_ptr(),
                                              _dt(w), topk, int(mode), out.data_ptr(), _dt(out), int(bool(accumulate)),
                                              ws.data_ptr(), ws.numel(), _stream_ptr(stream), ev))
        return out

    def forward_hc(self, x: torch.Tensor, sel: torch.Tensor, w: torch.Tensor, hc_x: torch.Tensor, post: torch.Tensor,
                   comb: torch.Tensor, y_half: bool = True, mode: int = _lib.MODE_EXACT, stream=None,
                   fn: torch.Tensor | None = None, partials: torch.Tensor | None = None) -> torch.Tensor:
        """The layer followed by the hyper-connection update of the MoE site (glmx_moe_forward_hc): hc_x fp32
        [ntok, 4, H] is updated in place with x_g <- post_g * y + sum_h comb[h][g] * x_h (y = the layer output, rounded
        to fp16 first when y_half); post fp32 [ntok, 4], comb fp32 [ntok, 4, 4]. Returns hc_x.
        With fn (fp16 [24, 4H]) and partials (fp32 [ntok, 4H/128, 25]) the next site's hc_mix_partials of the updated
        stack are written too (glmx_moe_forward_hc_mix; the reference's apply_partials, glm53/k_hcfuse.py:296-320)."""
        x = x.contiguous(); sel = sel.contiguous(); w = w.contiguous()
        ntok = x.shape[0]
        topk = sel.shape[1] if sel.dim() == 2 else 0
        if hc_x.shape != (ntok, 4, self.H) or hc_x.dtype != torch.float32 or not hc_x.is_contiguous():
            raise ValueError("hc_x must be contiguous fp32 [ntok, 4, H]")
        post = post.to(torch.float32).contiguous(); comb = comb.to(torch.float32).contiguous()
        if post.shape != (ntok, 4) or comb.shape != (ntok, 4, 4):
            raise ValueError("post must be [ntok, 4] and comb [ntok, 4, 4]")
        ws = self.workspace(ntok, topk)
        if fn is None:
            check(self.lib.glmx_moe_forward_hc(self.h, x.data_ptr(), _dt(x), ntok, sel.data_ptr(), _dt(sel), w.data_ptr(),
                                               _dt(w), topk, int(mode), hc_x.data_ptr(), post.data_ptr(), comb.data_ptr(),
                                               _lib.F16 if y_half else _lib.F32, ws.data_ptr(), ws.numel(),
                                               _stream_ptr(stream)))
            return hc_x
        from .hc import check_mix_args
        check_mix_args(hc_x, fn, partials)
        check(self.lib.glmx_moe_forward_hc_mix(self.h, x.data_ptr(), _dt(x), ntok, sel.data_ptr(), _dt(sel), w.data_ptr(),
                                               _dt(w), topk, int(mode), hc_x.data_ptr(), post.data_ptr(), comb.data_ptr(),
                                               _lib.F16 if y_half else _lib.F32, fn.data_ptr(), partials.data_ptr(),
                                               ws.data_ptr(), ws.numel(), _stream_ptr(stream)))
        return hc_x

    def forward_peer(self, x: torch.Tensor, sel: torch.Tensor, w: torch.Tensor, peer: "_lib.PeerOut",
                     mode: int = _lib.MODE_I16, stream=None) -> None:
        """The layer with the expert-parallel return (glmx_moe_forward_peer): each token's row goes to its owner
        rank's receive buffer instead of an output tensor (see glmx.ep)."""
        x = x.contiguous(); sel = sel.contiguous(); w = w.contiguous()
        ntok = x.shape[0]
        topk = sel.shape[1] if sel.dim() == 2 else 0
        ws = self.workspace(ntok, topk)
        check(self.lib.glmx_moe_forward_peer(self.h, x.data_ptr(), _dt(x), ntok, sel.data_ptr(), _dt(sel), w.data_ptr(),
                                             _dt(w), topk, int(mode), C.byref(peer), ws.data_ptr(), ws.numel(),
                                             _stream_ptr(stream)))

    def check_device(self, ntok: int, topk: int, stream=None) -> int:
        """Synchronise and read the device error word of the last call (0 = fine)."""
        flags = C.c_int(0)
        ws = self.workspace(ntok, topk)
        check(self.lib.glmx_check(self.h, int(ntok), int(topk), ws.data_ptr(), _stream_ptr(stream), C.byref(flags)))
        return flags.value


def decode_tiles(tiles: torch.Tensor, bits: int, stream=None) -> torch.Tensor:
    """Known-answer decode: uint8 CUDA tiles [n, 32*bits] -> fp16 bit patterns int16 [n, 16, 16]."""
    lib = _lib.load()
    tiles = tiles.contiguous()
    n = tiles.numel() // (32 * bits)
    out = torch.empty((n, 16, 16), dtype=torch.int16, device=tiles.device)
    check(lib.glmx_decode_tiles(tiles.data_ptr(), int(bits), n, out.data_ptr(), _stream_ptr(stream)))
    return out
