"""GPU parity of the expert-parallel pieces through the C ABI: uocr_moe_ep_experts (local experts
over received bf16 rows, entries without a local expert skipped), uocr_moe_shared_forward, and
ExpertParallelMoE end to end (one NCCL rank on one GPU; two ranks when two GPUs are visible),
against the float64 layer fed the bit-exact routing, at the prefill tolerance."""

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


def _ep_worker(rank: int, world: int, port: int, T: int, out_dir: str, kind: str) -> None:
    import sys

    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from oracle import moe_oracle as o

        uocr = importlib.import_module("unlimited-ocr-max_b200")
        ep = importlib.import_module("unlimited-ocr-max_b200.ep")
        cfg, w = full_layer(o, False, 4)
        placement = None
        if kind == "strided":  # every world-th expert, in descending order: local != global index
            placement = ep.ExpertPlacement([list(range(63 - p, -1, -world)) for p in range(world)])
        m = ep.ExpertParallelMoE(uocr.MoEConfig(), device=f"cuda:{rank}", placement=placement)
        m.load_state_dict(to_state(w, cfg, False))
        bias = np.random.default_rng(8).standard_normal(64).astype(np.float32)
        m.bias = torch.from_numpy(bias).to(f"cuda:{rank}")
        x = o.synth_hidden(T * world, cfg.hidden, 9)[rank * T:(rank + 1) * T]
        got = m(torch.from_numpy(x).to(f"cuda:{rank}"))
        np.save(os.path.join(out_dir, f"ep{rank}.npy"), got.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["contiguous", "strided"])
@pytest.mark.parametrize("world", [1, 2])
def test_expert_parallel_moe(oracle, tmp_path, world, kind):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    T = 512
    mp.spawn(_ep_worker, args=(world, _free_port(), T, str(tmp_path), kind), nprocs=world, join=True)
    got = np.concatenate([np.load(tmp_path / f"ep{r}.npy") for r in range(world)])
    cfg, w = full_layer(oracle, False, 4)
    bias = np.random.default_rng(8).standard_normal(64).astype(np.float32)
    x = oracle.synth_hidden(T * world, cfg.hidden, 9)
    r = oracle.route_fp32(x, w.router, bias, 6)
    _check(oracle, got, oracle.moe_layer_fp64(cfg, w, x, r.ids, r.weights))
