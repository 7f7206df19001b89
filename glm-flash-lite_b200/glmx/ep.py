"""Expert parallelism: the routed experts of one MoE layer sharded over the ranks of a process group.

Rank r of N holds routed experts [r*E/N, (r+1)*E/N) (a `MoELayer` with `first_expert = r*E/N`) and a copy of the
shared expert; every rank owns B tokens (the data-parallel part of the model gives each rank its own tokens). Per
layer call:

  dispatch   all-gather of the ranks' token rows x [B, H] and their routing (sel, w) [B, k] -> [N*B, ...]
  compute    the local shard over all N*B tokens: its picks only (other shards' ids are skipped by the split),
             weighted and summed per token into a partial [N*B, H] fp32 (tokens with no local pick get 0)
  return     reduce-scatter (sum) of the partials -> out [B, H] fp32 for this rank's own tokens
  shared     the shared expert over the rank's own B tokens, on a side stream while the dispatch is in flight,
             written into the rank's own rows of the partial before the local shard accumulates into it

With top-8 of 288 experts a token touches ≈ 5.3 of 8 shards, so gathering every token to every rank moves about as
many bytes as a per-destination all-to-all, with static sizes: no host synchronisation for split sizes, and the
collectives are the two NCCL has the best NVLink/NVSwitch paths for. The reference has no expert-parallel mode
(its experts run on one host's CPU cores); this is the multi-GPU form of its MoE layer (configs[3] of the build's
baseline: 288 experts over 2/4/8 GPUs).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(E: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous expert shard of `rank`: [first, first + count). E must divide evenly."""
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    n = E // world
    return rank * n, n


def _all_gather(out: torch.Tensor, inp: torch.Tensor, group) -> None:
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, inp, group=group)
    else:
        dist.all_gather(list(out.chunk(dist.get_world_size(group))), inp, group=group)


def _reduce_scatter(out: torch.Tensor, inp: torch.Tensor, group) -> None:
    if dist.get_backend(group) == "nccl":
        dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM, group=group)
    else:
        t = inp.clone()
        dist.all_reduce(t, group=group)
        out.copy_(t.chunk(dist.get_world_size(group))[dist.get_rank(group)])


class ExpertParallelLayer:
    """One MoE layer's routed experts sharded over `group` (see the module docstring).

    local: the rank's shard, an object with `forward(x, sel, w, mode=, out=, accumulate=)` over global expert ids
        (a `MoELayer` with `first_expert` set and no shared expert).
    shared: the shared expert as a one-expert layer (`MoELayer(E=1)`), or None.
    """

    def __init__(self, local, shared=None, group=None, E: int | None = None):
        self.local = local
        self.shared = shared
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = E
        self.device = getattr(local, "device", torch.device("cpu"))
        self._side = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self._bufs = {}

    def _buf(self, name, shape, dtype):
        b = self._bufs.get(name)
        if b is None or b.shape != shape or b.dtype != dtype:
            b = torch.empty(shape, dtype=dtype, device=self.device)
            self._bufs[name] = b
        return b

    def forward(self, x: torch.Tensor, sel: torch.Tensor, w: torch.Tensor, mode: int = 2,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """x [B, H] (same B on every rank), sel [B, k] global expert ids (< 0 = masked), w [B, k] -> out [B, H] fp32."""
        B, H = x.shape
        k = sel.shape[1]
        N, r = self.world, self.rank
        x = x.contiguous()
        sel = sel.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        partial = self._buf("partial", (N * B, H), torch.float32)
        main = torch.cuda.current_stream(self.device) if self._side is not None else None

        # shared expert over the own tokens, overlapping the dispatch
        if self._side is not None:
            self._side.wait_stream(main)
            ctx = torch.cuda.stream(self._side)
        else:
            ctx = _null()
        with ctx:
            partial.zero_()
            if self.shared is not None:
                ones_s = self._buf("sh_sel", (B, 1), torch.int32).zero_()
                ones_w = self._buf("sh_w", (B, 1), torch.float32).fill_(1.0)
                self.shared.forward(x, ones_s, ones_w, mode=mode, out=partial[r * B:(r + 1) * B], accumulate=False)

        # dispatch: token rows and routing of every rank
        xg = self._buf("xg", (N * B, H), x.dtype)
        _all_gather(xg, x, self.group)
        route = torch.cat([sel, w.view(torch.int32)], dim=1)
        rg = self._buf("rg", (N * B, 2 * k), torch.int32)
        _all_gather(rg, route, self.group)
        selg = rg[:, :k].contiguous()
        wg = rg[:, k:].contiguous().view(torch.float32)

        # compute: this shard's picks of all tokens, accumulated onto the shared rows
        if self._side is not None:
            main.wait_stream(self._side)
        self.local.forward(xg, selg, wg, mode=mode, out=partial, accumulate=True)

        # return: sum of the shards' partials, own rows
        if out is None:
            out = torch.empty((B, H), dtype=torch.float32, device=self.device)
        _reduce_scatter(out, partial, self.group)
        return out


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def from_bank(bank, group=None, device="cuda", act_limit: float = 0.0) -> ExpertParallelLayer:
    """This rank's shard of a synth.ExpertBank (+ its shared expert), uploaded to `device`."""
    import numpy as np

    from .layer import MoELayer

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    first, n = shard_range(bank.E, world, rank)
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())

    def upload(experts):
        parts = [bank.trellis[bank.proj_offset(e, 0):bank.proj_offset(e, 0) + bank.expert_bytes] for e in experts]
        tr = torch.from_numpy(np.concatenate(parts)).to(dev)
        ptrs = [[tr.data_ptr() + i * bank.expert_bytes + bank.proj_offset(e, p) - bank.proj_offset(e, 0)
                 for p in range(3)] for i, e in enumerate(experts)]
        suh = [torch.from_numpy(np.ascontiguousarray(s[experts])).to(dev) for s in bank.suh]
        svh = [torch.from_numpy(np.ascontiguousarray(s[experts])).to(dev) for s in bank.svh]
        return tr, ptrs, suh, svh

    tr, ptrs, suh, svh = upload(list(range(first, first + n)))
    local = MoELayer(bank.H, bank.I, n, ptrs, suh, svh, bits=bank.bits, has_shared=False, act_limit=act_limit,
                     keep=[tr], device=dev, first_expert=first)
    shared = None
    if bank.shared:
        tr_s, ptrs_s, suh_s, svh_s = upload([bank.E])
        shared = MoELayer(bank.H, bank.I, 1, ptrs_s, suh_s, svh_s, bits=bank.bits, has_shared=False,
                          act_limit=act_limit, keep=[tr_s], device=dev)
    return ExpertParallelLayer(local, shared, group, E=bank.E)
