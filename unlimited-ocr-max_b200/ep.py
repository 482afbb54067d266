"""Expert-parallel prefill of the MoE sublayer over P GPUs of one node.

The reference runs the MoE on one device; this is the B200 build's extension for large token
batches. Every rank holds T / P tokens, the replicated gate and shared experts, and E / P routed
experts, placed by an ``ExpertPlacement``: contiguous ranges by default (rank r owns experts
[r E/P, (r+1) E/P)), or balanced from measured expert loads (``balanced_placement``: a skewed
gate sends most rows to a few experts, and the rank holding them sets the step time). One
forward:

1. route the rank's tokens (the bit-exact gate, ``uocr_moe_route``);
2. plan: one row per (token, destination rank) that holds at least one of its k experts, rows
   ordered by destination rank, then token; each row carries, per slot, the expert's local index
   on that rank (or -1) and its routing weight;
3. exchange counts, then rows (bf16) and metadata, with ``all_to_all_single`` (NCCL over
   NVLink);
4. each rank applies its local experts to the rows it received, pre-weighted and summed per
   row (``uocr_moe_ep_experts``: the prefill's permute + tcgen05 grouped GEMMs);
5. exchange the fp32 partial rows back; each token sums its partials in destination-rank order
   (deterministic), then adds the sum of its shared experts (``uocr_moe_shared_forward``,
   data-parallel): out = (partial_0 + partial_1 + ...) + (shared_0 + shared_1).

``ep_forward`` states the bookkeeping (2, 3, 5) in plain torch; it runs on CPU ranks (gloo) in
the tests and is the reference the device path is checked against. ``ExpertParallelMoE`` runs
CUDA only: the plan and the bf16 row gather are one library call (``uocr_moe_ep_dispatch``, no
host round trip but the one D2H read of the exchanged row counts), the per-token sum of the
partials is another (``uocr_moe_ep_combine``), and the shared experts run on a side stream while
the rows are exchanged; the result is bit-identical to ``ep_forward`` with the same compute
steps.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Callable, Mapping

import torch
import torch.distributed as dist

from . import ops
from ._lib import check, load
from .moe import MoEConfig, UocrMoE

__all__ = ["ExpertPlacement", "contiguous_placement", "balanced_placement", "DispatchPlan", "plan_dispatch",
           "exchange_counts", "exchange_rows", "sum_partials", "ep_forward", "ExpertParallelMoE"]


@dataclass
class ExpertPlacement:
    """Which rank holds each routed expert: rank p holds ``experts[p]`` (global ids, the same
    number on every rank) as its local experts 0, 1, ... in that order."""

    experts: list[list[int]]
    _maps: dict = field(default_factory=dict, repr=False, compare=False)

    @property
    def world(self) -> int:
        return len(self.experts)

    @property
    def e_local(self) -> int:
        return len(self.experts[0])

    def owner_local(self, device=None) -> tuple[torch.Tensor, torch.Tensor]:
        """[E] int64 owner rank and [E] int64 local index of every expert (cached per device)."""
        key = str(torch.device(device) if device is not None else "cpu")
        if key not in self._maps:
            E = sum(len(v) for v in self.experts)
            owner = torch.empty(E, dtype=torch.int64)
            local = torch.empty(E, dtype=torch.int64)
            for p, ex in enumerate(self.experts):
                owner[ex] = p
                local[ex] = torch.arange(len(ex))
            self._maps[key] = (owner.to(device), local.to(device))
        return self._maps[key]


def contiguous_placement(E: int, world: int) -> ExpertPlacement:
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    n = E // world
    return ExpertPlacement([list(range(p * n, (p + 1) * n)) for p in range(world)])


def balanced_placement(load, world: int) -> ExpertPlacement:
    """E / world experts per rank with the routed rows (``load[e]``, e.g. a histogram of past
    routing decisions) spread as evenly as the greedy longest-first rule does it: experts by
    descending load (ties: lower id first) each go to the rank with the least load so far among
    those with room (ties: lower rank). Deterministic, so every rank computes the same map."""
    load = [int(v) for v in (load.tolist() if isinstance(load, torch.Tensor) else load)]
    E = len(load)
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    cap = E // world
    sums, experts = [0] * world, [[] for _ in range(world)]
    for e in sorted(range(E), key=lambda e: (-load[e], e)):
        p = min((q for q in range(world) if len(experts[q]) < cap), key=lambda q: (sums[q], q))
        experts[p].append(e)
        sums[p] += load[e]
    return ExpertPlacement([sorted(v) for v in experts])


def _as_placement(placement, world: int) -> ExpertPlacement:
    if isinstance(placement, ExpertPlacement):
        if placement.world != world:
            raise ValueError(f"placement for {placement.world} ranks used with {world}")
        return placement
    return contiguous_placement(int(placement) * world, world)  # an int: experts per rank, contiguous


@dataclass
class DispatchPlan:
    order: torch.Tensor        # [Ns] token of each send row (rows grouped by destination rank)
    send_counts: list[int]     # rows per destination rank
    meta_expert: torch.Tensor  # [Ns, k] int32: local expert index on the destination, -1 for none
    meta_weight: torch.Tensor  # [Ns, k] fp32 routing weight of the slot


def plan_dispatch(ids: torch.Tensor, wts: torch.Tensor, world: int, placement) -> DispatchPlan:
    """Rows to send: one per (token, destination rank) with at least one expert there.
    ``placement``: an ExpertPlacement, or an int (experts per rank, contiguous ranges)."""
    owner, local = _as_placement(placement, world).owner_local(ids.device)
    valid = ids >= 0  # id < 0: no expert in the slot
    idx = torch.where(valid, ids.long(), torch.zeros_like(ids.long()))
    dest = torch.where(valid, owner[idx], torch.full_like(idx, -1))  # [T, k]
    loc = local[idx]
    orders, counts, metas_e, metas_w = [], [], [], []
    for p in range(world):
        on_p = dest == p
        tok = torch.nonzero(on_p.any(dim=1), as_tuple=False).flatten()
        orders.append(tok)
        counts.append(int(tok.numel()))
        sel = on_p[tok]
        metas_e.append(torch.where(sel, loc[tok], torch.full_like(loc[tok], -1)).int())
        metas_w.append(torch.where(sel, wts[tok], torch.zeros_like(wts[tok])))
    return DispatchPlan(torch.cat(orders), counts, torch.cat(metas_e), torch.cat(metas_w))


def exchange_counts(send_counts: list[int], device, group=None) -> list[int]:
    world = len(send_counts)
    send = torch.tensor(send_counts, dtype=torch.int64, device=device)
    recv = torch.empty(world, dtype=torch.int64, device=device)
    dist.all_to_all_single(recv, send, group=group)
    return [int(v) for v in recv.tolist()]


def exchange_rows(t: torch.Tensor, send_counts: list[int], recv_counts: list[int], group=None) -> torch.Tensor:
    """all_to_all_single of the rows of ``t`` (rank p gets send_counts[p] rows, in order); with one
    rank the rows stay where they are."""
    if len(send_counts) == 1:
        return t
    out = torch.empty((sum(recv_counts),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, t.contiguous(), output_split_sizes=recv_counts, input_split_sizes=send_counts,
                           group=group)
    return out


def sum_partials(T: int, H: int, plan: DispatchPlan, partial: torch.Tensor) -> torch.Tensor:
    """out[t] = sum over destination ranks p (ascending) of the partial row of (t, p); every rank
    sends each token at most one row, so each step indexes distinct tokens (no atomics)."""
    out = torch.zeros((T, H), dtype=torch.float32, device=partial.device)
    r0 = 0
    for c in plan.send_counts:
        if c:
            out.index_add_(0, plan.order[r0:r0 + c], partial[r0:r0 + c])
        r0 += c
    return out


def ep_forward(x: torch.Tensor, route: Callable, local_experts: Callable, shared: Callable, world: int,
               placement, group=None) -> torch.Tensor:
    """One expert-parallel MoE forward of this rank's tokens x [T, H] fp32.

    route(x) -> (ids [T,k] int32 global, wts [T,k] fp32); local_experts(rows bf16 [N,H], meta_e,
    meta_w) -> fp32 [N,H] (meta_e: local expert indices); shared(x, buf) adds the shared experts
    into buf in place (given zeros). placement: as for plan_dispatch.
    """
    T, H = x.shape
    ids, wts = route(x)
    plan = plan_dispatch(ids, wts, world, placement)
    recv_counts = exchange_counts(plan.send_counts, x.device, group)
    rows = x.index_select(0, plan.order).to(torch.bfloat16)
    meta = torch.cat([plan.meta_expert, plan.meta_weight.view(torch.int32)], dim=1)  # one exchange
    rows_in = exchange_rows(rows, plan.send_counts, recv_counts, group)
    meta_in = exchange_rows(meta, plan.send_counts, recv_counts, group)
    k = ids.shape[1]
    part_in = local_experts(rows_in, meta_in[:, :k].contiguous(), meta_in[:, k:].contiguous().view(torch.float32))
    part = exchange_rows(part_in, recv_counts, plan.send_counts, group)
    out = sum_partials(T, H, plan, part)
    sh = torch.zeros_like(out)
    shared(x, sh)
    return out.add_(sh)  # routed + shared, the shared experts summed on their own first


class ExpertParallelMoE:
    """The MoE sublayer with its routed experts sharded over the ranks of ``group``.

    Construct on every rank after ``torch.distributed`` is initialised (backend "nccl"), with the
    same ``placement`` everywhere (default: contiguous ranges), load the full reference state dict
    (every rank keeps only its own routed experts), then call with the rank's tokens.
    """

    def __init__(self, config: MoEConfig, *, group=None, device: str | torch.device = "cuda",
                 placement: ExpertPlacement | None = None, overlap_shared: bool = True) -> None:
        self.config = config
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        E = config.n_routed_experts
        if E % self.world:
            raise ValueError(f"ExpertParallelMoE: {E} experts do not split over {self.world} ranks")
        if placement is None:
            placement = contiguous_placement(E, self.world)
        if placement.world != self.world or sorted(e for v in placement.experts for e in v) != list(range(E)) or \
                any(len(v) != E // self.world for v in placement.experts):
            raise ValueError("ExpertParallelMoE: placement must give every rank E / world distinct experts")
        self.placement = placement
        self.overlap_shared = overlap_shared
        self.e_local = E // self.world
        if self.e_local < config.num_experts_per_tok:
            raise ValueError("ExpertParallelMoE: fewer local experts than experts per token")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("ExpertParallelMoE runs on CUDA devices only")
        local_cfg = MoEConfig(**{**config.__dict__, "n_routed_experts": self.e_local})
        self.local = UocrMoE(local_cfg, device=self.device)
        self.router: torch.Tensor | None = None
        self.bias: torch.Tensor | None = None
        self._ws: dict[str, torch.Tensor] = {}
        self._bufs: dict[str, torch.Tensor] = {}
        self._phase_events: list | None = None
        owner, local = placement.owner_local(self.device)
        self._owner, self._local = owner.int().contiguous(), local.int().contiguous()
        self._side = torch.cuda.Stream(self.device)

    def load_state_dict(self, state: Mapping[str, torch.Tensor]) -> "ExpertParallelMoE":
        mine = torch.tensor(self.placement.experts[self.rank], dtype=torch.int64)
        local = {}
        for name, t in state.items():
            if name.startswith("experts."):
                t = t.index_select(0, mine.to(t.device))
            elif name == "gate.gate_score.weight":
                self.router = t.to(self.device, torch.bfloat16).contiguous()
                t = t[:self.e_local]  # unused by the local module (routing uses the full gate)
            local[name] = t
        self.local.load_state_dict(local)
        return self

    def check_status(self) -> None:
        """Synchronise and read (clearing) the device status of this rank's workspaces (the local
        experts', the shared experts' and the local module's): raises :class:`UocrError` if a
        device-side bounded wait gave up since the last check."""
        from ._lib import check as _check

        L = load()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        for name in ("ep", "shared"):
            ws = self._ws.get(name)
            if ws is not None:
                _check(L.uocr_moe_device_status(ws.data_ptr(), stream))
        self.local.check_status()

    def _workspace(self, name: str, nbytes: int) -> torch.Tensor:
        ws = self._ws.get(name)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._ws[name] = ws
        return ws

    def _buf(self, name: str, shape: tuple, dtype: torch.dtype) -> torch.Tensor:
        """A persistent buffer (reused across calls: the stream order keeps uses apart)."""
        n = 1
        for d in shape:
            n *= d
        b = self._bufs.get(name)
        if b is None or b.dtype != dtype or b.numel() < n:
            b = torch.empty(max(n, 1), dtype=dtype, device=self.device)
            self._bufs[name] = b
        return b[:n].view(shape)

    def _dispatch(self, x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor):
        """(send_counts int64 [world] on the device, rows bf16, meta int32 [.., 2k], inv int32 [world, T])."""
        T, H = x.shape
        k, W = ids.shape[1], self.world
        send = self._buf("send", (W,), torch.int64)
        rows = self._buf("rows", (T * W, H), torch.bfloat16)
        meta = self._buf("meta", (T * W, 2 * k), torch.int32)
        inv = self._buf("inv", (W, T), torch.int32)
        L = load()
        ws = self._workspace("dispatch", L.uocr_moe_ep_dispatch_workspace_bytes(T, W))
        check(L.uocr_moe_ep_dispatch(x.data_ptr(), T, H, ids.data_ptr(), wts.data_ptr(), k, self._owner.data_ptr(),
                                     self._local.data_ptr(), self.config.n_routed_experts, W, send.data_ptr(),
                                     rows.view(torch.int16).data_ptr(), meta.data_ptr(), inv.data_ptr(),
                                     ws.data_ptr(), ws.numel(), torch.cuda.current_stream(self.device).cuda_stream))
        return send, rows, meta, inv

    def _combine(self, part: torch.Tensor, inv: torch.Tensor, add: torch.Tensor | None, T: int) -> torch.Tensor:
        H = self.config.hidden_size
        out = torch.empty((T, H), dtype=torch.float32, device=self.device)
        check(load().uocr_moe_ep_combine(part.data_ptr(), part.shape[0], inv.data_ptr(), T, self.world, H,
                                         0 if add is None else add.data_ptr(), out.data_ptr(),
                                         torch.cuda.current_stream(self.device).cuda_stream))
        return out

    def _route(self, x: torch.Tensor):
        return ops.route(x, self.router, self.bias, self.config.num_experts_per_tok)

    def _local_experts(self, rows: torch.Tensor, meta_e: torch.Tensor, meta_w: torch.Tensor) -> torch.Tensor:
        N, H = rows.shape
        out = torch.empty((N, H), dtype=torch.float32, device=self.device)
        if N == 0:
            return out
        L = load()
        lay = ctypes.byref(self.local.layer)
        ws = self._workspace("ep", L.uocr_moe_ep_experts_workspace_bytes(lay, N))
        check(L.uocr_moe_ep_experts(lay, rows.view(torch.int16).data_ptr(), N, meta_e.data_ptr(), meta_w.data_ptr(),
                                    out.data_ptr(), ws.data_ptr(), ws.numel(),
                                    torch.cuda.current_stream(self.device).cuda_stream))
        return out

    def _shared(self, x: torch.Tensor, out: torch.Tensor, accumulate: int = 1) -> None:
        T = x.shape[0]
        if T == 0:
            return
        L = load()
        lay = ctypes.byref(self.local.layer)
        ws = self._workspace("shared", L.uocr_moe_shared_workspace_bytes(lay, T))
        check(L.uocr_moe_shared_forward(lay, x.data_ptr(), T, out.data_ptr(), accumulate, ws.data_ptr(), ws.numel(),
                                        torch.cuda.current_stream(self.device).cuda_stream))

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """The MoE over this rank's tokens x [T, H] fp32 (a collective: every rank calls it)."""
        if not x.is_cuda or x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != self.config.hidden_size:
            raise ValueError("ExpertParallelMoE: x must be a CUDA fp32 [T, hidden] tensor")
        x = x.contiguous()
        T, H = x.shape
        k, W, g = self.config.num_experts_per_tok, self.world, self.group
        cur = torch.cuda.current_stream(self.device)
        mark = self._mark
        mark("start")
        sh = self._buf("shared_out", (T, H), torch.float32)
        ids, wts = self._route(x)
        mark("route")
        send, rows, meta, inv = self._dispatch(x, ids, wts)
        mark("dispatch")
        # the shared experts overlap the exchanges (NCCL leaves most SMs free) or run in line
        if self.overlap_shared:
            self._side.wait_stream(cur)
            with torch.cuda.stream(self._side):
                self._shared(x, sh, accumulate=0)
        else:
            self._shared(x, sh, accumulate=0)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=g)
        counts = torch.cat([send, recv]).tolist()  # the one host synchronisation
        sc, rc = counts[:W], counts[W:]
        ns = sum(sc)
        mark("counts")
        rows_in = exchange_rows(rows[:ns], sc, rc, g)
        meta_in = exchange_rows(meta[:ns], sc, rc, g)
        mark("exchange_rows")
        part_in = self._local_experts(rows_in, meta_in[:, :k].contiguous(),
                                      meta_in[:, k:].contiguous().view(torch.float32))
        mark("experts")
        part = exchange_rows(part_in, rc, sc, g)
        mark("exchange_back")
        if self.overlap_shared:
            cur.wait_stream(self._side)
        mark("shared_wait")
        out = self._combine(part, inv, sh if T else None, T)
        mark("combine")
        return out

    def _mark(self, name: str) -> None:
        if self._phase_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self._phase_events.append((name, ev))

    def profile_phases(self, x: torch.Tensor, steps: int = 10) -> dict[str, float]:
        """Mean device time (ms) between the phase boundaries of ``steps`` calls on this rank's
        main stream: route, dispatch, counts (exchange + the host read), exchange_rows,
        experts, exchange_back, shared_wait (the side stream's shared experts not yet done),
        combine. A collective: every rank calls it."""
        acc: dict[str, float] = {}
        for _ in range(steps):
            self._phase_events = []
            self(x)
            torch.cuda.synchronize(self.device)
            evs, self._phase_events = self._phase_events, None
            for (_, a), (name, b) in zip(evs, evs[1:]):
                acc[name] = acc.get(name, 0.0) + a.elapsed_time(b) / steps
        return {k: round(v, 4) for k, v in acc.items()}

    def forward_reference(self, x: torch.Tensor) -> torch.Tensor:
        """The same layer through the torch bookkeeping of ``ep_forward`` (the device path's check)."""
        return ep_forward(x.contiguous(), self._route, self._local_experts, self._shared, self.world,
                          self.placement, self.group)
