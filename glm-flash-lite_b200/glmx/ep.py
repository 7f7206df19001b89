"""Expert parallelism: the routed experts of one MoE layer sharded over the ranks of a process group.

Rank r of N holds routed experts [r*E/N, (r+1)*E/N) and a copy of the shared expert, in ONE `MoELayer` of n + 1
experts (the shard at local ids 0..n-1, the shared expert at local id n); every rank owns B tokens (the data-parallel
part of the model gives each rank its own tokens). Per layer call:

  dispatch   all-gather of the ranks' token rows x [B, H] and their routing (sel, w) [B, k] -> [N*B, ...]
  split      global ids -> local ids of this shard (others' ids masked to -1), plus one extra pick per row: the
             shared expert (local id n, weight 1) for the rank's own B rows, masked for the other ranks' rows
  compute    one layer call over all N*B rows: its picks only, weighted and summed per row into a partial [N*B, H]
             fp32 (rows with no local pick get 0); the shared expert rides in the same launches as a routed expert
  return     reduce-scatter (sum) of the partials -> out [B, H] fp32 for this rank's own rows

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

    local: the rank's layer, an object with `forward(x, sel, w, mode=, out=, accumulate=)` over LOCAL expert ids
        0..n-1 (the shard's experts first .. first + n - 1) and, when `has_shared`, local id n = the shared expert
        (a `MoELayer` with n + 1 experts, `has_shared=False`).
    first, n: the shard's expert range. E: routed experts of the whole layer.
    """

    def __init__(self, local, first: int, n: int, has_shared: bool = True, group=None, E: int | None = None):
        self.local = local
        self.first, self.n, self.has_shared = int(first), int(n), bool(has_shared)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = E
        self.device = getattr(local, "device", torch.device("cpu"))
        self._bufs = {}

    def _buf(self, name, shape, dtype):
        b = self._bufs.get(name)
        if b is None or b.shape != shape or b.dtype != dtype:
            b = torch.empty(shape, dtype=dtype, device=self.device)
            self._bufs[name] = b
        return b

    def _extra(self, NB: int, B: int):
        """the shared-expert pick column: local id n with weight 1 on this rank's own rows, -1 / 0 elsewhere"""
        key = ("extra", NB, B)
        if key not in self._bufs:
            own = torch.zeros(NB, dtype=torch.bool, device=self.device)
            own[self.rank * B:(self.rank + 1) * B] = True
            s = torch.where(own, self.n, -1).to(torch.int32).reshape(NB, 1)
            self._bufs[key] = (s.contiguous(), own.to(torch.float32).reshape(NB, 1).contiguous())
        return self._bufs[key]

    def forward(self, x: torch.Tensor, sel: torch.Tensor, w: torch.Tensor, mode: int = 2,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """x [B, H] (same B on every rank), sel [B, k] global expert ids (< 0 = masked), w [B, k] -> out [B, H] fp32."""
        B, H = x.shape
        k = sel.shape[1]
        N = self.world
        x = x.contiguous()
        sel = sel.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()

        # dispatch: token rows and routing of every rank
        xg = self._buf("xg", (N * B, H), x.dtype)
        _all_gather(xg, x, self.group)
        route = torch.cat([sel, w.view(torch.int32)], dim=1)
        rg = self._buf("rg", (N * B, 2 * k), torch.int32)
        _all_gather(rg, route, self.group)

        # split: this shard's local ids (+ the shared expert on the own rows)
        loc = rg[:, :k] - self.first
        loc = torch.where((loc >= 0) & (loc < self.n), loc, torch.full_like(loc, -1))
        wl = rg[:, k:].view(torch.float32)
        if self.has_shared:
            es, ew = self._extra(N * B, B)
            loc = torch.cat([loc, es], dim=1)
            wl = torch.cat([wl, ew], dim=1)
        loc = loc.contiguous()
        wl = wl.contiguous()

        # compute: this shard's picks of all rows (+ shared on the own rows), one layer call
        partial = self._buf("partial", (N * B, H), torch.float32)
        self.local.forward(xg, loc, wl, mode=mode, out=partial, accumulate=False)

        # return: sum of the shards' partials, own rows
        if out is None:
            out = torch.empty((B, H), dtype=torch.float32, device=self.device)
        _reduce_scatter(out, partial, self.group)
        return out


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

    experts = list(range(first, first + n)) + ([bank.E] if bank.shared else [])
    tr, ptrs, suh, svh = upload(experts)
    local = MoELayer(bank.H, bank.I, len(experts), ptrs, suh, svh, bits=bank.bits, has_shared=False, act_limit=act_limit,
                     keep=[tr], device=dev)
    return ExpertParallelLayer(local, first, n, has_shared=bank.shared, group=group, E=bank.E)
