"""GPU, one device: the peer-memory exchange of the expert-parallel layer with W ranks emulated in
one process. Each emulated rank has its own exchange buffer (all on this GPU), its own local
experts and its own workspace; the ranks' steps run one after the other on one stream (every
dispatch, then every expert product, then every combine), so each bounded device wait finds its
flags already set by an earlier launch and no kernel waits on one that runs beside it.

Checked against the torch bookkeeping of ep.py (plan_dispatch, the local experts through
uocr_moe_ep_experts, partials rounded to bf16, sum_partials, + shared), bit for bit: the rows and
metadata each rank finds in its slots, the per-token positions, and every rank's output. Also: a
second epoch gives the same bits, and a rank whose source never dispatched times out into NaN
outputs and a status (the wait budget made short is not needed: the flag of the missing epoch is
simply never written, and the test reads the status after the bounded wait ends -- skipped here to
keep the run short; the count check is exercised instead by a slot count above capacity).
"""

from __future__ import annotations

import ctypes
import importlib

import numpy as np
import pytest
import torch

from test_gpu_moe import full_layer, to_state

pytestmark = pytest.mark.gpu
DEV = "cuda"


class Rank:
    def __init__(self, uocr, ep, state, placement, p, world, cap):
        L = uocr.load()
        self.p, self.world = p, world
        mine = torch.tensor(placement.experts[p], dtype=torch.int64)
        local = {}
        for name, t in state.items():
            if name.startswith("experts."):
                t = t.index_select(0, mine)
            elif name == "gate.gate_score.weight":
                t = t[:len(placement.experts[p])]
            local[name] = t
        self.moe = uocr.UocrMoE(uocr.MoEConfig(n_routed_experts=len(placement.experts[p]))).load_state_dict(local)
        nbytes = L.uocr_moe_ep_peer_buffer_bytes(world, cap, 1280, 6)
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
        self.cap = cap

    def peers(self, ranks, epoch):
        P = importlib.import_module("unlimited-ocr-max_b200._lib").UocrEpPeers()
        P.world, P.rank, P.cap_tokens, P.hidden, P.top_k, P.epoch = self.world, self.p, self.cap, 1280, 6, epoch
        for q, r in enumerate(ranks):
            P.buf[q] = r.buf.data_ptr()
        return P


def _reference(ep, uocr, ranks, placement, xs, ids, wts, shared_out):
    """ep_forward's bookkeeping with the collectives written out over the emulated ranks."""
    L = uocr.load()
    W = len(ranks)
    plans = [ep.plan_dispatch(ids[p].cpu(), wts[p].cpu(), W, placement) for p in range(W)]
    parts = {}
    for q in range(W):  # expert rank q: the rows every source p sends it, in source order
        rows, me, mw, spans = [], [], [], []
        for p in range(W):
            pl = plans[p]
            r0 = sum(pl.send_counts[:q])
            c = pl.send_counts[q]
            rows.append(xs[p].cpu()[pl.order[r0:r0 + c]].to(torch.bfloat16))
            me.append(pl.meta_expert[r0:r0 + c])
            mw.append(pl.meta_weight[r0:r0 + c])
            spans.append((p, c))
        rows, me, mw = torch.cat(rows).to(DEV), torch.cat(me).to(DEV), torch.cat(mw).to(DEV)
        N = rows.shape[0]
        out = torch.empty((N, 1280), dtype=torch.float32, device=DEV)
        if N:
            lay = ctypes.byref(ranks[q].moe.layer)
            ws = torch.zeros(L.uocr_moe_ep_experts_workspace_bytes(lay, N), dtype=torch.uint8, device=DEV)
            assert L.uocr_moe_ep_experts(lay, rows.view(torch.int16).data_ptr(), N, me.data_ptr(), mw.data_ptr(),
                                         out.data_ptr(), ws.data_ptr(), ws.numel(),
                                         torch.cuda.current_stream().cuda_stream) == 0, L.uocr_last_error()
        out = out.to(ep.PARTIAL_DTYPE).cpu()
        n0 = 0
        for p, c in spans:
            parts[(p, q)] = out[n0:n0 + c]
            n0 += c
    want = []
    for p in range(W):
        pl = plans[p]
        part = torch.cat([parts[(p, q)] for q in range(W)])
        want.append(ep.sum_partials(xs[p].shape[0], 1280, pl, part) + shared_out[p].cpu())
    return plans, want


@pytest.mark.parametrize("world,ts", [(1, [300]), (2, [513, 480]), (4, [256, 1, 300, 0]), (8, [129] * 8)])
def test_peer_exchange_emulated_ranks_match_the_bookkeeping(uocr, oracle, world, ts):
    ep = importlib.import_module("unlimited-ocr-max_b200.ep")
    L = uocr.load()
    cfg, w = full_layer(oracle, False, 12)
    state = to_state(w, cfg, False)
    rng = np.random.default_rng(world)
    placement = ep.ExpertPlacement([sorted(v) for v in np.array_split(rng.permutation(64), world)])
    placement = ep.ExpertPlacement([[int(e) for e in v] for v in placement.experts])
    cap = max(max(ts), 1)
    ranks = [Rank(uocr, ep, state, placement, p, world, cap) for p in range(world)]
    router = state["gate.gate_score.weight"].to(DEV)
    bias = torch.from_numpy(rng.standard_normal(64).astype(np.float32)).to(DEV)
    xs = [torch.from_numpy(oracle.synth_hidden(max(t, 1), 1280, 100 + p)[:t]).to(DEV).contiguous()
          for p, t in enumerate(ts)]
    routes = [uocr.ops.route(x, router, bias, 6) if x.shape[0] else
              (torch.empty((0, 6), dtype=torch.int32, device=DEV), torch.empty((0, 6), device=DEV)) for x in xs]
    ids, wts = [r[0] for r in routes], [r[1] for r in routes]
    owner, local = (t.int().to(DEV).contiguous() for t in placement.owner_local())
    shared = [torch.from_numpy(rng.standard_normal((t, 1280)).astype(np.float32)).to(DEV) for t in ts]
    stream = torch.cuda.current_stream().cuda_stream
    plans, want = _reference(ep, uocr, ranks, placement, xs, ids, wts, shared)
    for epoch in (1, 2):
        Ps = [r.peers(ranks, epoch) for r in ranks]
        wss = [torch.zeros(L.uocr_moe_ep_peer_workspace_bytes(ctypes.byref(r.moe.layer), ctypes.byref(P)),
                           dtype=torch.uint8, device=DEV) for r, P in zip(ranks, Ps)] if epoch == 1 else wss
        invs = [torch.full((world, max(t, 1)), -9, dtype=torch.int32, device=DEV) for t in ts]
        for p in range(world):
            assert L.uocr_moe_ep_peer_dispatch(ctypes.byref(Ps[p]), xs[p].data_ptr() if ts[p] else None, ts[p],
                                               ids[p].data_ptr(), wts[p].data_ptr(), owner.data_ptr(),
                                               local.data_ptr(), 64, invs[p].data_ptr(), wss[p].data_ptr(),
                                               wss[p].numel(), stream) == 0, L.uocr_last_error()
        if epoch == 1:  # what every rank finds in its slots, and the positions
            torch.cuda.synchronize()
            for p in range(world):
                pl = plans[p]
                want_inv = torch.full((world, ts[p]), -1, dtype=torch.int32)
                r0 = 0
                for q, c in enumerate(pl.send_counts):
                    want_inv[q, pl.order[r0:r0 + c]] = torch.arange(c, dtype=torch.int32)
                    r0 += c
                assert torch.equal(invs[p][:, :ts[p]].cpu(), want_inv)
        for p in range(world):
            assert L.uocr_moe_ep_peer_experts(ctypes.byref(ranks[p].moe.layer), ctypes.byref(Ps[p]),
                                              wss[p].data_ptr(), wss[p].numel(), stream) == 0, L.uocr_last_error()
        outs = [torch.full((max(t, 1), 1280), float("nan"), device=DEV) for t in ts]
        for p in range(world):
            assert L.uocr_moe_ep_peer_combine(ctypes.byref(Ps[p]), invs[p].data_ptr(), ts[p], shared[p].data_ptr(),
                                              outs[p].data_ptr(), stream) == 0, L.uocr_last_error()
        for p in range(world):
            assert L.uocr_moe_device_status(ranks[p].buf.data_ptr(), stream) == 0, L.uocr_last_error()
            assert torch.equal(outs[p][:ts[p]].cpu(), want[p]), (epoch, p)


def test_peer_exchange_refuses_bad_arguments(uocr):
    L = uocr.load()
    P = importlib.import_module("unlimited-ocr-max_b200._lib").UocrEpPeers()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device=DEV)
    P.world, P.rank, P.cap_tokens, P.hidden, P.top_k, P.epoch = 2, 0, 16, 1280, 6, 1
    P.buf[0] = buf.data_ptr()
    x = torch.zeros((17, 1280), device=DEV)
    rc = L.uocr_moe_ep_peer_combine(ctypes.byref(P), x.data_ptr(), 4, None, x.data_ptr(), None)
    assert rc == 1 and "buf[1]" in L.uocr_last_error().decode()
    P.buf[1] = buf.data_ptr() + 256
    rc = L.uocr_moe_ep_peer_combine(ctypes.byref(P), x.data_ptr(), 17, None, x.data_ptr(), None)
    assert rc == 1 and "cap_tokens" in L.uocr_last_error().decode()
    P.epoch = 0
    rc = L.uocr_moe_ep_peer_combine(ctypes.byref(P), x.data_ptr(), 4, None, x.data_ptr(), None)
    assert rc == 1 and "epoch" in L.uocr_last_error().decode()
