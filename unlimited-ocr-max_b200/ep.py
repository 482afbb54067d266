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
3. send the rows (bf16) and their metadata to the destination ranks;
4. each rank applies its local experts to the rows it received, pre-weighted and summed per
   row (the prefill's permute + tcgen05 grouped GEMMs), rounded to bf16;
5. send the partial rows back; each token sums its partials in destination-rank order
   (deterministic), then adds the sum of its shared experts (``uocr_moe_shared_forward``,
   data-parallel): out = (partial_0 + partial_1 + ...) + (shared_0 + shared_1).

``ExpertParallelMoE`` (exchange "peer", the default) does 2-5 in three library calls with no
all-to-all and no host synchronisation: every rank maps every other rank's exchange buffer (CUDA
IPC, plain peer loads and stores over NVLink, no multicast), the dispatch kernels store the rows
and metadata straight into the destinations' slots, the expert products store the partial rows
straight back, and per-source epoch flags written with system-scope release order the two sides
(bounded device waits; a failure gives NaN outputs and a status that ``check_status`` raises).
``ep_forward`` states the same bookkeeping in plain torch over ``torch.distributed`` collectives
(the count table, ``all_to_all_single`` of rows, metadata and partials); it runs on CPU ranks
(gloo) in the tests, serves exchange "nccl", and is the reference the peer path is checked
against bit for bit. Its host-side exchanges take a timeout: a rank that does not take part in
time, or a count table that cannot be right, raises :class:`ExchangeError` on every rank that
sees it, after aborting the communicator, before any rows move.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from datetime import timedelta
from typing import Callable, Mapping

import torch
import torch.distributed as dist

from . import ops
from ._lib import UocrEpPeers, check, load
from .moe import MoEConfig, UocrMoE

__all__ = ["ExpertPlacement", "contiguous_placement", "balanced_placement", "DispatchPlan", "plan_dispatch",
           "ExchangeError", "count_table", "exchange_counts", "exchange_rows", "sum_partials", "ep_forward",
           "ExpertParallelMoE", "PARTIAL_DTYPE"]

#: dtype of the partial rows the expert ranks send back (half the bytes of fp32; the rounding is far
#: inside the layer's tolerance)
PARTIAL_DTYPE = torch.bfloat16
#: default time a rank waits for the others at a host-side exchange
DEFAULT_TIMEOUT_S = 120.0


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


class ExchangeError(RuntimeError):
    """An expert-parallel exchange failed on the host: a rank did not take part within the timeout,
    or the exchanged row counts cannot be right. Raised on every rank that sees it."""


def _abort(group) -> None:
    """Abort the NCCL communicator so that no later collective waits on a rank that is gone (other
    backends have no abort: their next collective times out on its own)."""
    try:
        if dist.get_backend(group) == "nccl":
            dist.distributed_c10d._abort_process_group(group)
    except Exception:  # noqa: BLE001 - the ExchangeError raised next is what matters
        pass


def _wait(work, what: str, timeout_s: float | None, group) -> None:
    """Wait for an async collective at most ``timeout_s`` seconds on the host (None: no limit)."""
    if timeout_s is None:
        work.wait()
        return
    try:
        done = work.wait(timeout=timedelta(seconds=timeout_s))
    except Exception as e:  # noqa: BLE001 - the backends raise RuntimeError on a timeout
        _abort(group)
        raise ExchangeError(f"{what}: not every rank took part within {timeout_s:g} s ({e})") from e
    if done is False:
        _abort(group)
        raise ExchangeError(f"{what}: not every rank took part within {timeout_s:g} s")


def count_table(send_counts: list[int], T: int, device, group=None, timeout_s: float | None = None) -> torch.Tensor:
    """Every rank's row counts and token count, gathered (host tensor [world, world + 1]: row p is
    rank p's rows to ranks 0..world-1, then its T). Every rank gets the same table and checks it the
    same way, so a bad count is refused by every rank before any row moves: a count below 0 or above
    the sender's token count (a rank sends each token at most one row per destination)."""
    world = dist.get_world_size(group)
    mine = torch.tensor([*send_counts, T], dtype=torch.int64, device=device)
    parts = [torch.empty_like(mine) for _ in range(world)]
    _wait(dist.all_gather(parts, mine, group=group, async_op=True), "row counts", timeout_s, group)
    tab = torch.stack(parts).cpu()
    if tab.shape != (world, world + 1):
        raise ExchangeError(f"row counts: a rank sent {tab.shape[1] - 1} counts for {world} ranks")
    for p in range(world):
        tp = int(tab[p, world])
        for q in range(world):
            c = int(tab[p, q])
            if c < 0 or c > tp:
                raise ExchangeError(f"row counts: rank {p} announces {c} rows for rank {q} from {tp} tokens")
    return tab


def exchange_counts(send_counts: list[int], device, group=None, T: int | None = None,
                    timeout_s: float | None = None) -> list[int]:
    """The rows this rank receives from each rank (from the checked count table)."""
    rank = dist.get_rank(group)
    tab = count_table(send_counts, max(send_counts) if T is None else T, device, group, timeout_s)
    return [int(v) for v in tab[:, rank].tolist()]


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
            out.index_add_(0, plan.order[r0:r0 + c], partial[r0:r0 + c].float())
        r0 += c
    return out


def ep_forward(x: torch.Tensor, route: Callable, local_experts: Callable, shared: Callable, world: int,
               placement, group=None, timeout_s: float | None = DEFAULT_TIMEOUT_S) -> torch.Tensor:
    """One expert-parallel MoE forward of this rank's tokens x [T, H] fp32.

    route(x) -> (ids [T,k] int32 global, wts [T,k] fp32); local_experts(rows bf16 [N,H], meta_e,
    meta_w) -> fp32 [N,H] (meta_e: local expert indices), sent back rounded to PARTIAL_DTYPE;
    shared(x, buf) adds the shared experts into buf in place (given zeros). placement: as for
    plan_dispatch. The count exchange waits at most ``timeout_s`` (None: no limit) and refuses an
    impossible count table (:class:`ExchangeError`) before any row moves.
    """
    T, H = x.shape
    ids, wts = route(x)
    plan = plan_dispatch(ids, wts, world, placement)
    recv_counts = exchange_counts(plan.send_counts, x.device, group, T=T, timeout_s=timeout_s)
    rows = x.index_select(0, plan.order).to(torch.bfloat16)
    meta = torch.cat([plan.meta_expert, plan.meta_weight.view(torch.int32)], dim=1)  # one exchange
    rows_in = exchange_rows(rows, plan.send_counts, recv_counts, group)
    meta_in = exchange_rows(meta, plan.send_counts, recv_counts, group)
    k = ids.shape[1]
    part_in = local_experts(rows_in, meta_in[:, :k].contiguous(), meta_in[:, k:].contiguous().view(torch.float32))
    part = exchange_rows(part_in.to(PARTIAL_DTYPE), recv_counts, plan.send_counts, group)
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
                 placement: ExpertPlacement | None = None, overlap_shared: bool = True, exchange: str = "peer",
                 timeout_s: float | None = DEFAULT_TIMEOUT_S, max_tokens: int | None = None) -> None:
        """``exchange``: "peer" (stores into the other ranks' memory, no host synchronisation; the
        default) or "nccl" (``ep_forward``'s collectives, one host read of the count table).
        ``timeout_s`` bounds every host-side wait on the other ranks (the set-up of the peer
        buffers, the "nccl" count exchange): past it the communicator is aborted and
        :class:`ExchangeError` raised. ``max_tokens``: the most tokens any rank passes in one call
        (default: the largest T of the first call, agreed by all ranks)."""
        if exchange not in ("peer", "nccl"):
            raise ValueError(f"ExpertParallelMoE: exchange {exchange!r} (peer or nccl)")
        self.exchange = exchange
        self.timeout_s = timeout_s
        self.max_tokens = max_tokens
        self._peer: dict | None = None
        self._epoch = 0
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
        if self._peer is not None:
            _check(L.uocr_moe_device_status(self._peer["own"].data_ptr(), stream))
        self.local.check_status()

    # ---- the peer exchange ------------------------------------------------------------------
    def _setup_peers(self, T: int) -> None:
        """Collective (every rank, at its first call): agree on the slot capacity, allocate this
        rank's exchange buffer, and map every other rank's (CUDA IPC handles all-gathered)."""
        L, g, W = load(), self.group, self.world
        cap = torch.tensor([T if self.max_tokens is None else self.max_tokens], dtype=torch.int64, device=self.device)
        _wait(dist.all_reduce(cap, op=dist.ReduceOp.MAX, group=g, async_op=True), "exchange set-up", self.timeout_s, g)
        cap = int(cap.item())
        H, k = self.config.hidden_size, self.config.num_experts_per_tok
        nbytes = L.uocr_moe_ep_peer_buffer_bytes(W, cap, H, k)
        if nbytes == 0:
            raise ValueError(f"ExpertParallelMoE: no exchange buffer for {W} ranks x {cap} tokens")
        own = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)  # epochs and flags start at 0
        torch.cuda.synchronize(self.device)
        handle = (ctypes.c_ubyte * 64)()
        off = ctypes.c_uint64()
        check(L.uocr_ipc_export(own.data_ptr(), ctypes.cast(handle, ctypes.c_void_p), ctypes.byref(off)))
        mine = torch.tensor(list(bytes(handle)) + list(int(off.value).to_bytes(8, "little")), dtype=torch.uint8,
                            device=self.device)
        parts = [torch.empty_like(mine) for _ in range(W)]
        _wait(dist.all_gather(parts, mine, group=g, async_op=True), "exchange set-up", self.timeout_s, g)
        P = UocrEpPeers()
        P.world, P.rank, P.cap_tokens, P.hidden, P.top_k = W, self.rank, cap, H, k
        imported = []
        for q, t in enumerate(parts):
            if q == self.rank:
                P.buf[q] = own.data_ptr()
                continue
            b = bytes(t.cpu().tolist())
            h = (ctypes.c_ubyte * 64).from_buffer_copy(b[:64])
            o = int.from_bytes(b[64:], "little")
            ptr = ctypes.c_void_p()
            check(L.uocr_ipc_import(ctypes.cast(h, ctypes.c_void_p), o, ctypes.byref(ptr)))
            P.buf[q] = ptr.value
            imported.append((ptr.value, o))
        _wait(dist.barrier(group=g, async_op=True), "exchange set-up", self.timeout_s, g)
        self._peer = {"P": P, "own": own, "imported": imported, "cap": cap}

    def close(self) -> None:
        """Unmap the other ranks' exchange buffers (after the stream's work is done)."""
        if self._peer is not None:
            torch.cuda.synchronize(self.device)
            L = load()
            for ptr, o in self._peer["imported"]:
                L.uocr_ipc_close(ptr, o)
            self._peer = None

    def _call_peer(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        if self._peer is None:
            self._setup_peers(T)
        pe = self._peer
        if T > pe["cap"]:
            raise ValueError(f"ExpertParallelMoE: {T} tokens, above the exchange capacity {pe['cap']} "
                             "(construct with max_tokens)")
        P = pe["P"]
        self._epoch += 1
        P.epoch = self._epoch
        L = load()
        lay = ctypes.byref(self.local.layer)
        cur = torch.cuda.current_stream(self.device)
        stream = cur.cuda_stream
        mark = self._mark
        mark("start")
        sh = self._buf("shared_out", (T, H), torch.float32)
        ids, wts = self._route(x)
        mark("route")
        inv = self._buf("inv", (self.world, T), torch.int32)
        ws = self._workspace("peer", L.uocr_moe_ep_peer_workspace_bytes(lay, ctypes.byref(P)))
        check(L.uocr_moe_ep_peer_dispatch(ctypes.byref(P), x.data_ptr(), T, ids.data_ptr(), wts.data_ptr(),
                                          self._owner.data_ptr(), self._local.data_ptr(),
                                          self.config.n_routed_experts, inv.data_ptr(), ws.data_ptr(), ws.numel(),
                                          stream))
        mark("dispatch")
        if self.overlap_shared:
            self._side.wait_stream(cur)
            with torch.cuda.stream(self._side):
                self._shared(x, sh, accumulate=0)
        else:
            self._shared(x, sh, accumulate=0)
        check(L.uocr_moe_ep_peer_experts(lay, ctypes.byref(P), ws.data_ptr(), ws.numel(), stream))
        mark("experts")
        if self.overlap_shared:
            cur.wait_stream(self._side)
        mark("shared_wait")
        out = torch.empty((T, H), dtype=torch.float32, device=self.device)
        check(L.uocr_moe_ep_peer_combine(ctypes.byref(P), inv.data_ptr(), T, sh.data_ptr() if T else None,
                                         out.data_ptr(), stream))
        mark("combine")
        return out

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
        if self.exchange == "peer":
            return self._call_peer(x)
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
        tab = count_table(send.tolist(), T, self.device, g, self.timeout_s)  # the one host synchronisation
        sc, rc = tab[self.rank, :W].tolist(), tab[:, self.rank].tolist()
        ns = sum(sc)
        mark("counts")
        rows_in = exchange_rows(rows[:ns], sc, rc, g)
        meta_in = exchange_rows(meta[:ns], sc, rc, g)
        mark("exchange_rows")
        part_in = self._local_experts(rows_in, meta_in[:, :k].contiguous(),
                                      meta_in[:, k:].contiguous().view(torch.float32))
        mark("experts")
        part = exchange_rows(part_in.to(PARTIAL_DTYPE), rc, sc, g).float()
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
        main stream. Exchange "peer": route, dispatch (plan; rows and metadata stored into the
        destinations), experts (wait for every source; expert products; partial rows stored back),
        shared_wait (the side stream's shared experts not yet done), combine (wait for every expert
        rank; sum). Exchange "nccl": route, dispatch, counts (count table + the host read),
        exchange_rows, experts, exchange_back, shared_wait, combine. A collective: every rank
        calls it."""
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
                          self.placement, self.group, self.timeout_s)
