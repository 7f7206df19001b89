"""Expert parallelism: the routed experts of one MoE layer sharded over the ranks of a process group.

Rank r of N holds routed experts [r*E/N, (r+1)*E/N) and a copy of the shared expert, in ONE `MoELayer` of n + 1
experts (the shard at local ids 0..n-1, the shared expert at local id n); every rank owns B tokens (the data-parallel
part of the model gives each rank its own tokens). Two exchanges.

exchange="a2a": per destination, only the tokens with a pick there travel.

  shared     the shared expert on the rank's own rows, on a side stream, while the exchange below is in flight
  pack       glmx_ep_pack: per destination rank, its tokens (ascending), their rows and their picks in the
             destination's local ids (one kernel; counts per destination)
  dispatch   all-to-all of the counts, then (one host synchronisation for the split sizes) all-to-all of the rows and
             of their routing
  compute    one layer call over the received rows (this shard's picks only)
  return     all-to-all of the fp32 results back to the token owners, in the order they were sent; glmx_ep_unpack_add
             adds each token's returned rows in rank order onto the shared expert's output

exchange="allgather" (the default; and "peer"):

  dispatch   all-gather of the ranks' token rows x [B, H] and their routing (sel, w) [B, k] -> [N*B, ...]
  split      global ids -> local ids of this shard (others' ids masked to -1), plus one extra pick per row: the
             shared expert (local id n, weight 1) for the rank's own B rows, masked for the other ranks' rows
  compute    one layer call over all N*B rows: its picks only, weighted and summed per row into a partial [N*B, H]
             fp32 (rows with no local pick get 0); the shared expert rides in the same launches as a routed expert
  return     reduce-scatter (sum) of the partials -> out [B, H] fp32 for the rank's own rows; or, with peer=True on
             NCCL groups of GPUs, the combine itself stores each token's partial row into its owner rank's receive
             buffer over peer memory (NVLink / NVSwitch; CUDA IPC mappings made once) and flags the owner, which sums
             the N partials in rank order (glmx_moe_forward_peer + glmx_peer_reduce)

With top-8 of 288 experts a token touches ≈ 5.3 of 8 shards, so gathering every token to every rank moves about as
many bytes as a per-destination all-to-all, with static sizes: no host synchronisation for split sizes. The split is one
kernel (glmx_ep_split). At decode sizes that wins: on 2 B200s at global B=64 the all-to-all's dispatch (count
exchange, host synchronisation for NCCL's split sizes, rows and routing) takes 0.191 ms against the all-gather's 0.038
ms, for rows of 12 KB each, so "allgather" is the default and "a2a" the form for batches whose rows, not latency,
dominate. Measured on 8 B200s at global B=64 (one layer, an earlier build): 161.7 K tok/s with NCCL's reduce-scatter,
157.2 K with the peer-memory return; NCCL reduces inside the NVSwitch (NVLS) and so moves half the bytes the
point-to-point stores of the fused return do, which is why the reduce-scatter is the default return. The reference has no expert-parallel mode
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


class _PeerReturn:
    """Receive buffers, flags and their peer mappings for the expert-parallel return of B rows per rank (one set per
    layer and B). Made collectively: every rank of the group builds it in the same call."""

    def __init__(self, group, device, world: int, rank: int, B: int, H: int):
        import ctypes as C

        from . import _lib
        L = _lib.load()
        self.L, self.world, self.rank, self.B, self.H = L, world, rank, B, H
        self.seq = 0
        self.own = []
        self.opened = []

        def alloc(nbytes):
            p = C.c_void_p()
            _lib.check(L.glmx_ipc_alloc(nbytes, C.byref(p)))
            self.own.append(p.value)
            return p.value

        self.recv = alloc(4 * 2 * world * B * H)          # float [2][world][B][H], written by every rank
        self.flags = alloc(4 * 2 * world)                 # int [2][world], written by every rank
        self.local_words = torch.zeros(2, dtype=torch.int32, device=device)   # [arrival counter, error word]

        def handle(ptr):
            h = (C.c_char * _lib.IPC_HANDLE_BYTES)()
            _lib.check(L.glmx_ipc_handle(ptr, h))
            return bytes(h)

        mine = (handle(self.recv), handle(self.flags))
        hs = [None] * world
        dist.all_gather_object(hs, mine, group=group)
        recv_tab, flag_tab = [], []
        for d in range(world):
            if d == rank:
                recv_tab.append(self.recv); flag_tab.append(self.flags)
                continue
            pr, pf = C.c_void_p(), C.c_void_p()
            _lib.check(L.glmx_ipc_open(hs[d][0], C.byref(pr)))
            self.opened.append(pr.value)
            _lib.check(L.glmx_ipc_open(hs[d][1], C.byref(pf)))
            self.opened.append(pf.value)
            recv_tab.append(pr.value); flag_tab.append(pf.value)
        self.tabs = torch.tensor([recv_tab, flag_tab], dtype=torch.int64, device=device)
        dist.barrier(group=group)

    def peer_out(self):
        from . import _lib
        if not hasattr(self, "_po"):
            self._po = _lib.PeerOut(self.tabs[0].data_ptr(), self.tabs[1].data_ptr(), self.local_words.data_ptr(), self.rank,
                                    self.world, self.B, 0)
        self.seq += 1
        self._po.seq = self.seq
        return self._po

    def reduce(self, out: torch.Tensor, stream=None) -> None:
        from . import _lib
        from .layer import _stream_ptr
        _lib.check(self.L.glmx_peer_reduce(self.recv, self.flags, self.world, self.B, self.H, self.seq, out.data_ptr(),
                                           _lib.F32 if out.dtype == torch.float32 else _lib.F16,
                                           self.local_words.data_ptr() + 4, _stream_ptr(stream)))

    def error_flags(self) -> int:
        """the return's device error word (16: a peer's flag did not come within the wait limit); synchronises"""
        return int(self.local_words[1].item())

    def close(self) -> None:
        for p in self.opened:
            self.L.glmx_ipc_close(p)
        self.opened = []
        for p in self.own:
            self.L.glmx_ipc_free(p)
        self.own = []


class ExpertParallelLayer:
    """One MoE layer's routed experts sharded over `group` (see the module docstring).

    local: the rank's layer, an object with `forward(x, sel, w, mode=, out=, accumulate=)` over LOCAL expert ids
        0..n-1 (the shard's experts first .. first + n - 1) and, when `has_shared`, local id n = the shared expert
        (a `MoELayer` with n + 1 experts, `has_shared=False`).
    first, n: the shard's expert range. E: routed experts of the whole layer.
    """

    def __init__(self, local, first: int, n: int, has_shared: bool = True, group=None, E: int | None = None,
                 peer: bool = False, exchange: str = "allgather"):
        self.local = local
        self.first, self.n, self.has_shared = int(first), int(n), bool(has_shared)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = E
        self.device = getattr(local, "device", torch.device("cpu"))
        self._bufs = {}
        # peer-memory return (on request): NCCL groups of GPU ranks, when the local layer has the peer entry (MoELayer)
        can = dist.get_backend(group) == "nccl" and self.device.type == "cuda" and hasattr(local, "forward_peer")
        if peer and not can:
            raise ValueError("the peer-memory return needs an NCCL group of GPU ranks and a MoELayer shard")
        self.peer = bool(peer)
        self.exchange = "peer" if self.peer else exchange
        if self.exchange not in ("a2a", "allgather", "peer"):
            raise ValueError("exchange must be 'a2a', 'allgather' or 'peer'")
        self._ret = None
        self._side = None
        self.events = None        # optional 4 torch.cuda.Event: start, dispatch done, compute done, return done

    def close(self) -> None:
        """Release the peer mappings (collective: every rank calls it; before destroy_process_group)."""
        if self._ret is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self._ret.close()
            self._ret = None

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

    def forward(self, x: torch.Tensor, sel: torch.Tensor, w: torch.Tensor, mode: int = 1,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """x [B, H] (same B on every rank), sel [B, k] global expert ids (< 0 = masked), w [B, k] -> out [B, H] fp32."""
        B, H = x.shape
        k = sel.shape[1]
        N = self.world
        x = x.contiguous()
        sel = sel.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        if self.exchange == "a2a":
            return self._forward_a2a(x, sel, w, mode, out)
        self._mark(0)

        # dispatch: token rows and routing of every rank
        xg = self._buf("xg", (N * B, H), x.dtype)
        _all_gather(xg, x, self.group)
        route = torch.cat([sel, w.view(torch.int32)], dim=1)
        rg = self._buf("rg", (N * B, 2 * k), torch.int32)
        _all_gather(rg, route, self.group)

        # split: this shard's local ids (+ the shared expert on the own rows)
        kk = k + (1 if self.has_shared else 0)
        if self.device.type == "cuda" and hasattr(self.local, "lib"):
            from . import _lib
            from .layer import _stream_ptr
            loc = self._buf("loc", (N * B, kk), torch.int32)
            wl = self._buf("wl", (N * B, kk), torch.float32)
            _lib.check(self.local.lib.glmx_ep_split(rg.data_ptr(), N * B, k, self.first, self.n, int(self.has_shared),
                                                    self.rank * B, (self.rank + 1) * B, loc.data_ptr(), wl.data_ptr(),
                                                    _stream_ptr(None)))
        else:
            loc = rg[:, :k] - self.first
            loc = torch.where((loc >= 0) & (loc < self.n), loc, torch.full_like(loc, -1))
            wl = rg[:, k:].view(torch.float32)
            if self.has_shared:
                es, ew = self._extra(N * B, B)
                loc = torch.cat([loc, es], dim=1)
                wl = torch.cat([wl, ew], dim=1)
            loc = loc.contiguous()
            wl = wl.contiguous()

        if out is None:
            out = torch.empty((B, H), dtype=torch.float32, device=self.device)
        if self.peer:
            # compute + return: the combine stores each row's partial into its owner's receive slot (peer memory);
            # the owner adds the N partials of its rows in rank order once their flags are in
            if self._ret is None or self._ret.B != B or self._ret.H != H:
                if self._ret is not None:
                    self.close()
                self._ret = _PeerReturn(self.group, self.device, N, self.rank, B, H)
            po = self._ret.peer_out()
            self.local.forward_peer(xg, loc, wl, po, mode=mode)
            self._ret.reduce(out)
            return out

        # compute: this shard's picks of all rows (+ shared on the own rows), one layer call
        self._mark(1)
        partial = self._buf("partial", (N * B, H), torch.float32)
        self.local.forward(xg, loc, wl, mode=mode, out=partial, accumulate=False)
        self._mark(2)

        # return: sum of the shards' partials, own rows
        _reduce_scatter(out, partial, self.group)
        self._mark(3)
        return out


    # ---- all-to-all exchange ----------------------------------------------------------------------------------------
    def _mark(self, i):
        if self.events is not None and self.device.type == "cuda":
            self.events[i].record(torch.cuda.current_stream(self.device))

    def _pack(self, x, sel, w):
        """(counts [N] int32, send_tok, send_route [., 2k] int32, pos [N, B] int32, send_x) in (destination, token) order."""
        B, H = x.shape
        k = sel.shape[1]
        N, n = self.world, self.n
        if self.device.type == "cuda" and hasattr(self.local, "lib"):
            from . import _lib
            from .layer import _stream_ptr
            cnt = self._buf("a2a_counts", (N + 1,), torch.int32)
            send_tok = self._buf("a2a_tok", (max(1, N * B),), torch.int32)
            send_route = self._buf("a2a_route", (max(1, N * B), 2 * k), torch.int32)
            pos = self._buf("a2a_pos", (N, max(1, B)), torch.int32)
            send_x = self._buf("a2a_x", (max(1, N * B), H), x.dtype)
            _lib.check(self.local.lib.glmx_ep_pack(sel.data_ptr(), w.data_ptr(), B, k, n, N, x.data_ptr(), H * x.element_size(),
                                                   cnt.data_ptr(), cnt.data_ptr() + 4 * N, send_tok.data_ptr(),
                                                   send_route.data_ptr(), pos.data_ptr(), send_x.data_ptr(), _stream_ptr(None)))
            return cnt[:N], send_tok, send_route, pos, send_x
        # the same order with tensor operations (CPU process groups: the host-logic tests)
        owner = torch.where(sel >= 0, torch.div(sel, n, rounding_mode="floor"), torch.full_like(sel, -1))
        mask = torch.zeros((N, B), dtype=torch.bool, device=x.device)
        for j in range(k):
            ok = (owner[:, j] >= 0) & (owner[:, j] < N)
            mask[owner[ok, j].long(), torch.arange(B, device=x.device)[ok]] = True
        d_idx, t_idx = mask.nonzero(as_tuple=True)
        counts = mask.sum(dim=1).to(torch.int32)
        pos = torch.full((N, B), -1, dtype=torch.int32, device=x.device)
        pos[d_idx, t_idx] = torch.arange(d_idx.numel(), dtype=torch.int32, device=x.device)
        s = sel[t_idx]
        mine = owner[t_idx] == d_idx[:, None]
        loc = torch.where(mine, s - d_idx[:, None].to(s.dtype) * n, torch.full_like(s, -1))
        wl = torch.where(mine, w[t_idx], torch.zeros_like(w[t_idx]))
        route = torch.cat([loc, wl.view(torch.int32)], dim=1).contiguous()
        return counts, t_idx.to(torch.int32), route, pos, x[t_idx].contiguous()

    def _forward_a2a(self, x, sel, w, mode, out):
        B, H = x.shape
        k = sel.shape[1]
        N = self.world
        cuda = self.device.type == "cuda"
        self._mark(0)
        if out is None:
            out = torch.empty((B, H), dtype=torch.float32, device=self.device)
        # the shared expert on the own rows does not wait for the exchange: a side stream runs it meanwhile
        side_done = None
        if self.has_shared:
            ssel = self._buf(("sh_sel", B), (B, 1), torch.int32)
            sw = self._buf(("sh_w", B), (B, 1), torch.float32)
            ssel.fill_(self.n)
            sw.fill_(1.0)
            if cuda:
                if self._side is None:
                    self._side = torch.cuda.Stream(self.device)
                    self._side_ws = None
                ready = torch.cuda.Event()
                ready.record(torch.cuda.current_stream(self.device))
                self._side.wait_event(ready)
                with torch.cuda.stream(self._side):
                    need = self.local.workspace_bytes(B, 1)
                    if self._side_ws is None or self._side_ws.numel() < need:
                        self._side_ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=self.device)
                    self.local.forward(x, ssel, sw, mode=mode, out=out, workspace=self._side_ws)
                    side_done = torch.cuda.Event()
                    side_done.record(self._side)
            else:
                self.local.forward(x, ssel, sw, mode=mode, out=out)
        else:
            out.zero_()
        counts, send_tok, send_route, pos, send_x = self._pack(x, sel, w)
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        c = torch.stack([counts, recv_counts]).cpu()           # split sizes on the host (one synchronisation)
        sc, rc = [int(v) for v in c[0]], [int(v) for v in c[1]]
        S, R = sum(sc), sum(rc)
        cap = max(1, N * B)                                    # a source sends each rank at most its B rows
        recv_x = self._buf("a2a_rx", (cap, H), x.dtype)[:R]
        recv_route = self._buf("a2a_rr", (cap, 2 * k), torch.int32)[:R]
        dist.all_to_all_single(recv_x, send_x[:S], rc, sc, group=self.group)
        dist.all_to_all_single(recv_route, send_route[:S], rc, sc, group=self.group)
        self._mark(1)
        # this shard's picks of the received rows
        partial = self._buf("a2a_part", (cap, H), torch.float32)[:R]
        if R:
            self.local.forward(recv_x, recv_route[:, :k], recv_route[:, k:].view(torch.float32), mode=mode, out=partial)
        self._mark(2)
        # return: the results go back to the token owners in the order they were sent
        ret = self._buf("a2a_ret", (cap, H), torch.float32)[:S]
        dist.all_to_all_single(ret, partial, sc, rc, group=self.group)
        if side_done is not None:
            torch.cuda.current_stream(self.device).wait_event(side_done)
        if cuda and hasattr(self.local, "lib"):
            from . import _lib
            from .layer import _stream_ptr
            _lib.check(self.local.lib.glmx_ep_unpack_add(ret.data_ptr(), pos.data_ptr(), B, N, H, out.data_ptr(), _stream_ptr(None)))
        else:
            for d in range(N):
                p = pos[d]
                has = p >= 0
                out[has] += ret[p[has].long()]
        self._mark(3)
        return out


def from_bank(bank, group=None, device="cuda", act_limit: float = 0.0, peer: bool = False,
              exchange: str = "allgather") -> ExpertParallelLayer:
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
    return ExpertParallelLayer(local, first, n, has_shared=bank.shared, group=group, E=bank.E, peer=peer, exchange=exchange)
