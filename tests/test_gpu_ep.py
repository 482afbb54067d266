"""GPU parity of the expert-parallel pieces through the C ABI: uocr_moe_ep_experts (local experts
over received bf16 rows, entries without a local expert skipped), uocr_moe_shared_forward, and
ExpertParallelMoE end to end, with the peer-memory exchange and with the NCCL bookkeeping, on 1, 2,
4 and 8 ranks (one process per GPU; the cases with more ranks than visible GPUs are skipped),
against the float64 layer fed the bit-exact routing, at the prefill tolerance. The dispatch and
combine kernels (uocr_moe_ep_dispatch / uocr_moe_ep_combine) must reproduce the torch
bookkeeping of ep.py bit for bit, and so must the whole device path of either exchange."""

from __future__ import annotations

import ctypes
import importlib
import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_gpu_moe import full_layer, to_state

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = Path(__file__).resolve().parents[1]


def _check(oracle, got, ref):
    assert np.all(np.isfinite(got))
    assert np.max(np.abs(got - ref)) <= 2e-2, np.max(np.abs(got - ref))
    assert oracle.rel_l2(got, ref) <= 1e-2, oracle.rel_l2(got, ref)


def _stacks(oracle, w):
    return {n: oracle.bf16_to_f32(getattr(w, n)).astype(np.float64) for n in ("gate", "up", "down")}


def _layer(uocr, oracle):
    cfg, w = full_layer(oracle, False, 3)
    moe = uocr.UocrMoE(uocr.MoEConfig()).load_state_dict(to_state(w, cfg, False))
    return cfg, w, moe


def test_ep_experts_vs_fp64(uocr, oracle):
    cfg, w, moe = _layer(uocr, oracle)
    L = uocr.load()
    lay = ctypes.byref(moe.layer)
    st = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(5)
    N = 300
    x = oracle.synth_hidden(N, cfg.hidden, 6)
    rows = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    meta_e = rng.integers(-1, 64, (N, 6)).astype(np.int32)
    meta_w = rng.random((N, 6)).astype(np.float32)
    de, dw = torch.from_numpy(meta_e).to(DEV), torch.from_numpy(meta_w).to(DEV)
    out = torch.empty((N, cfg.hidden), dtype=torch.float32, device=DEV)
    ws = torch.zeros(L.uocr_moe_ep_experts_workspace_bytes(lay, N), dtype=torch.uint8, device=DEV)
    rc = L.uocr_moe_ep_experts(lay, rows.view(torch.int16).data_ptr(), N, de.data_ptr(), dw.data_ptr(), out.data_ptr(),
                               ws.data_ptr(), ws.numel(), st)
    assert rc == 0, L.uocr_last_error()
    assert L.uocr_moe_device_status(ws.data_ptr(), st) == 0, L.uocr_last_error()
    xb = rows.float().cpu().numpy().astype(np.float64)
    s = _stacks(oracle, w)
    silu = lambda a: a / (1.0 + np.exp(-a))  # noqa: E731
    ref = np.zeros_like(xb)
    for e in range(64):
        nn, ss = np.nonzero(meta_e == e)
        if nn.size:
            xe = xb[nn]
            y = (silu(xe @ s["gate"][e].T) * (xe @ s["up"][e].T)) @ s["down"][e].T
            np.add.at(ref, nn, meta_w[nn, ss][:, None] * y)
    _check(oracle, out.cpu().numpy(), ref)


def _random_routing(rng, T, k, E, none_frac=0.1):
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32) if T else np.zeros((0, k), np.int32)
    ids[rng.random((T, k)) < none_frac] = -1
    wts = rng.random((T, k)).astype(np.float32)
    return ids, wts


def _dispatch(L, x, ids, wts, placement, world):
    T, H = x.shape
    k = ids.shape[1]
    owner, local = (t.int().to(DEV).contiguous() for t in placement.owner_local())
    send = torch.full((world,), -7, dtype=torch.int64, device=DEV)
    rows = torch.zeros((max(T * world, 1), H), dtype=torch.bfloat16, device=DEV)
    meta = torch.zeros((max(T * world, 1), 2 * k), dtype=torch.int32, device=DEV)
    inv = torch.zeros((world, max(T, 1)), dtype=torch.int32, device=DEV)
    ws = torch.zeros(max(L.uocr_moe_ep_dispatch_workspace_bytes(T, world), 1), dtype=torch.uint8, device=DEV)
    rc = L.uocr_moe_ep_dispatch(x.data_ptr(), T, H, ids.data_ptr(), wts.data_ptr(), k, owner.data_ptr(),
                                local.data_ptr(), owner.numel(), world, send.data_ptr(),
                                rows.view(torch.int16).data_ptr(), meta.data_ptr(), inv.data_ptr(), ws.data_ptr(),
                                ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.uocr_last_error()
    return send, rows, meta, inv


@pytest.mark.parametrize("world,T", [(1, 300), (2, 1), (2, 257), (3, 1000), (4, 4096), (8, 513), (4, 0)])
def test_ep_dispatch_matches_torch_plan(uocr, world, T):
    ep = importlib.import_module("unlimited-ocr-max_b200.ep")
    L = uocr.load()
    rng = np.random.default_rng(world * 1000 + T)
    E, k, H = 64, 6, 1280
    perm = rng.permutation(E)
    placement = ep.ExpertPlacement([sorted(perm[p::world].tolist()) for p in range(world)])
    ids_np, wts_np = _random_routing(rng, T, k, E)
    ids, wts = torch.from_numpy(ids_np).to(DEV), torch.from_numpy(wts_np).to(DEV)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32) * 3).to(DEV)
    send, rows, meta, inv = _dispatch(L, x, ids, wts, placement, world)
    plan = ep.plan_dispatch(ids.cpu(), wts.cpu(), world, placement)
    assert send.cpu().tolist() == plan.send_counts
    ns = sum(plan.send_counts)
    assert torch.equal(rows[:ns].cpu().view(torch.int16), x.cpu()[plan.order].to(torch.bfloat16).view(torch.int16))
    assert torch.equal(meta[:ns, :k].cpu(), plan.meta_expert)
    assert torch.equal(meta[:ns, k:].cpu(), plan.meta_weight.view(torch.int32))
    want_inv = torch.full((world, T), -1, dtype=torch.int32)
    r0 = 0
    for p, c in enumerate(plan.send_counts):
        want_inv[p, plan.order[r0:r0 + c]] = torch.arange(r0, r0 + c, dtype=torch.int32)
        r0 += c
    assert torch.equal(inv[:, :T].cpu(), want_inv)


@pytest.mark.parametrize("with_add", [False, True])
def test_ep_combine_matches_sum_partials(uocr, with_add):
    ep = importlib.import_module("unlimited-ocr-max_b200.ep")
    L = uocr.load()
    rng = np.random.default_rng(3)
    world, T, E, k, H = 4, 777, 64, 6, 1280
    placement = ep.balanced_placement(rng.integers(0, 1000, E), world)
    ids_np, wts_np = _random_routing(rng, T, k, E, 0.3)
    ids, wts = torch.from_numpy(ids_np).to(DEV), torch.from_numpy(wts_np).to(DEV)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(DEV)
    send, rows, meta, inv = _dispatch(L, x, ids, wts, placement, world)
    plan = ep.plan_dispatch(ids.cpu(), wts.cpu(), world, placement)
    ns = sum(plan.send_counts)
    part = torch.from_numpy(rng.standard_normal((ns, H)).astype(np.float32)).to(DEV)
    add = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(DEV) if with_add else None
    out = torch.full((T, H), float("nan"), device=DEV)
    rc = L.uocr_moe_ep_combine(part.data_ptr(), ns, inv.data_ptr(), T, world, H, 0 if add is None else add.data_ptr(),
                               out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.uocr_last_error()
    want = ep.sum_partials(T, H, plan, part.cpu())
    if add is not None:
        want = want + add.cpu()
    assert torch.equal(out.cpu(), want)


@pytest.mark.parametrize("accumulate", [0, 1])
def test_shared_forward_vs_fp64(uocr, oracle, accumulate):
    cfg, w, moe = _layer(uocr, oracle)
    L = uocr.load()
    lay = ctypes.byref(moe.layer)
    st = torch.cuda.current_stream().cuda_stream
    N = 300
    x = oracle.synth_hidden(N, cfg.hidden, 6)
    base = torch.from_numpy(np.random.default_rng(7).standard_normal((N, cfg.hidden)).astype(np.float32)).to(DEV)
    acc = base.clone()
    ws = torch.zeros(L.uocr_moe_shared_workspace_bytes(lay, N), dtype=torch.uint8, device=DEV)
    xt = torch.from_numpy(x).to(DEV)
    assert L.uocr_moe_shared_forward(lay, xt.data_ptr(), N, acc.data_ptr(), accumulate, ws.data_ptr(), ws.numel(),
                                     st) == 0, L.uocr_last_error()
    assert L.uocr_moe_device_status(ws.data_ptr(), st) == 0, L.uocr_last_error()
    silu = lambda a: a / (1.0 + np.exp(-a))  # noqa: E731
    sg, su, sd = (oracle.bf16_to_f32(a).astype(np.float64) for a in (w.shared_gate, w.shared_up, w.shared_down))
    xf = x.astype(np.float64)
    ref = (silu(xf @ sg.T) * (xf @ su.T)) @ sd.T
    got = (acc - base).cpu().numpy() if accumulate else acc.cpu().numpy()
    _check(oracle, got, ref)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _token_split(T: int, world: int, kind: str) -> list[int]:
    """Tokens per rank: equal, or ragged (rank r has 37 r fewer)."""
    return [T - 37 * r for r in range(world)] if kind == "ragged" else [T] * world


def _ep_worker(rank: int, world: int, port: int, T: int, out_dir: str, kind: str, exchange: str) -> None:
    import sys

    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    m = None
    try:
        from oracle import moe_oracle as o

        uocr = importlib.import_module("unlimited-ocr-max_b200")
        ep = importlib.import_module("unlimited-ocr-max_b200.ep")
        cfg, w = full_layer(o, False, 4)
        placement = None
        if kind == "strided":  # every world-th expert, in descending order: local != global index
            placement = ep.ExpertPlacement([list(range(63 - p, -1, -world)) for p in range(world)])
        m = ep.ExpertParallelMoE(uocr.MoEConfig(), device=f"cuda:{rank}", placement=placement,
                                 overlap_shared=kind != "strided", exchange=exchange, timeout_s=120)
        m.load_state_dict(to_state(w, cfg, False))
        bias = np.random.default_rng(8).standard_normal(64).astype(np.float32)
        m.bias = torch.from_numpy(bias).to(f"cuda:{rank}")
        ts = _token_split(T, world, kind)
        x = o.synth_hidden(sum(ts), cfg.hidden, 9)[sum(ts[:rank]):sum(ts[:rank + 1])]
        xd = torch.from_numpy(x).to(f"cuda:{rank}")
        got = m(xd)
        # the device exchange reproduces the torch bookkeeping of ep_forward bit for bit
        assert torch.equal(got, m.forward_reference(xd))
        assert torch.equal(got, m(xd))
        ph = m.profile_phases(xd, 2)
        want = (["route", "dispatch", "experts", "shared_wait", "combine"] if exchange == "peer" else
                ["route", "dispatch", "counts", "exchange_rows", "experts", "exchange_back", "shared_wait", "combine"])
        assert list(ph) == want and all(v >= 0 for v in ph.values())
        assert torch.equal(m(xd), got)  # after the phase calls (later epochs) still the same bits
        m.check_status()
        np.save(os.path.join(out_dir, f"ep{rank}.npy"), got.cpu().numpy())
        dist.barrier()
    finally:
        if m is not None:
            m.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
@pytest.mark.parametrize("kind", ["contiguous", "strided", "ragged"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_expert_parallel_moe(oracle, tmp_path, world, kind, exchange):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    if kind == "ragged" and world == 1:
        pytest.skip("one rank: nothing to be ragged against")
    T = 512
    mp.spawn(_ep_worker, args=(world, _free_port(), T, str(tmp_path), kind, exchange), nprocs=world, join=True)
    got = np.concatenate([np.load(tmp_path / f"ep{r}.npy") for r in range(world)])
    cfg, w = full_layer(oracle, False, 4)
    bias = np.random.default_rng(8).standard_normal(64).astype(np.float32)
    x = oracle.synth_hidden(sum(_token_split(T, world, kind)), cfg.hidden, 9)
    r = oracle.route_fp32(x, w.router, bias, 6)
    _check(oracle, got, oracle.moe_layer_fp64(cfg, w, x, r.ids, r.weights))
