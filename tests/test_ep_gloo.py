"""Expert-parallel bookkeeping on CPU ranks (gloo, world sizes 2 and 4): the dispatch plan, the count
and row exchanges and the per-token sum of partials, with the expert compute done by a float64
restatement of the layer on the receiving rank. The gathered outputs of all ranks must equal
the single-process float64 layer (routing from the bit-exact fp32 oracle) to the prefill
tolerance (the rows travel as bf16, as in the CUDA path)."""

from __future__ import annotations

import importlib
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
H, I, E, K, S = 256, 128, 8, 6, 2
T_TOTAL = 48


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup():
    sys.path.insert(0, str(ROOT))
    from oracle import moe_oracle as o

    cfg = o.MoEConfig(hidden=H, inter=I, n_routed=E, n_shared=S, top_k=K)
    w = o.synth_weights(cfg, 11, std=0.05)
    x = o.synth_hidden(T_TOTAL, H, 12)
    return o, cfg, w, x


def _placement(ep, world: int, kind: str):
    if kind == "contiguous":
        return E // world
    # balanced from a skewed histogram: the hot experts 0 and 1 land on different ranks
    return ep.balanced_placement([90, 80, 10, 10, 5, 5, 1, 1], world)


def _worker(rank: int, world: int, port: int, out_dir: str, kind: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ep = importlib.import_module("unlimited-ocr-max_b200.ep")
        o, cfg, w, x = _setup()
        placement = _placement(ep, world, kind)
        experts = ep.contiguous_placement(E, world).experts if kind == "contiguous" else placement.experts
        t_local = T_TOTAL // world
        xl = torch.from_numpy(x[rank * t_local:(rank + 1) * t_local].copy())
        st = {n: o.bf16_to_f32(getattr(w, n)).astype(np.float64) for n in ("gate", "up", "down")}
        sg, su, sd = (o.bf16_to_f32(a).astype(np.float64) for a in (w.shared_gate, w.shared_up, w.shared_down))
        silu = lambda a: a / (1.0 + np.exp(-a))  # noqa: E731

        def route(xt):
            r = o.route_fp32(xt.numpy(), w.router, None, K)
            return torch.from_numpy(r.ids), torch.from_numpy(r.weights)

        def local_experts(rows, meta_e, meta_w):
            xr = rows.float().numpy().astype(np.float64)
            out = np.zeros_like(xr)
            for n in range(xr.shape[0]):
                for s in range(K):
                    e = int(meta_e[n, s])
                    if e < 0:
                        continue
                    g = experts[rank][e]
                    hcol = silu(st["gate"][g] @ xr[n]) * (st["up"][g] @ xr[n])
                    out[n] += float(meta_w[n, s]) * (st["down"][g] @ hcol)
            return torch.from_numpy(out.astype(np.float32))

        def shared(xt, out):
            xf = xt.numpy().astype(np.float64)
            out += torch.from_numpy(((silu(xf @ sg.T) * (xf @ su.T)) @ sd.T).astype(np.float32))

        got = ep.ep_forward(xl, route, local_experts, shared, world, placement)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), got.numpy())
    finally:
        dist.destroy_process_group()


def test_plan_dispatch_rows_and_metadata():
    ep = importlib.import_module("unlimited-ocr-max_b200.ep")
    ids = torch.tensor([[0, 5, 1, 7, 2, 3], [4, 5, 6, 7, 0, 1], [0, 1, 2, 3, 4, 5]], dtype=torch.int32)
    wts = torch.arange(18, dtype=torch.float32).view(3, 6) / 100
    plan = ep.plan_dispatch(ids, wts, 2, 4)
    assert plan.send_counts == [3, 3]  # every token has experts on both ranks
    assert plan.order.tolist() == [0, 1, 2, 0, 1, 2]
    # token 0 on rank 1: experts 5 and 7 -> local 1 and 3 in slots 1 and 3
    assert plan.meta_expert[3].tolist() == [-1, 1, -1, 3, -1, -1]
    assert torch.equal(plan.meta_weight[3], torch.tensor([0, 0.01, 0, 0.03, 0, 0]))
    one = ep.plan_dispatch(torch.tensor([[0, 1, 2, 3, 0, 1]], dtype=torch.int32), wts[:1], 2, 4)
    assert one.send_counts == [1, 0]


def test_balanced_placement():
    ep = importlib.import_module("unlimited-ocr-max_b200.ep")
    pl = ep.balanced_placement([90, 80, 10, 10, 5, 5, 1, 1], 2)
    assert pl.experts == [[0, 3, 6, 7], [1, 2, 4, 5]]  # loads 102 and 100
    owner, local = pl.owner_local()
    assert owner.tolist() == [0, 1, 1, 0, 1, 1, 0, 0] and local.tolist() == [0, 0, 1, 1, 2, 3, 2, 3]
    # Zipf-skewed loads over 64 experts on 4 ranks: expert 0 alone exceeds the mean rank load,
    # so the best any placement can do is expert 0 plus the 15 lightest; the greedy rule gets
    # that, where contiguous ranges put the whole head on rank 0
    load = [int(1e6 / (e + 1) ** 1.1) for e in range(64)]
    worst = max(sum(load[e] for e in v) for v in ep.balanced_placement(load, 4).experts)
    assert worst == load[0] + sum(sorted(load)[:15])
    assert max(sum(load[16 * p:16 * p + 16]) for p in range(4)) > 2 * worst
    with pytest.raises(ValueError):
        ep.balanced_placement([1] * 7, 2)


def test_plan_dispatch_with_placement():
    ep = importlib.import_module("unlimited-ocr-max_b200.ep")
    pl = ep.ExpertPlacement([[0, 2, 4, 6], [1, 3, 5, 7]])
    ids = torch.tensor([[0, 5, 1, 7, 2, 3]], dtype=torch.int32)
    plan = ep.plan_dispatch(ids, torch.ones(1, 6), 2, pl)
    assert plan.send_counts == [1, 1]
    assert plan.meta_expert.tolist() == [[0, -1, -1, -1, 1, -1], [-1, 2, 0, 3, -1, 1]]
    # id -1 (no expert) sends nothing, to no rank
    none = ep.plan_dispatch(torch.tensor([[-1, -1, 1, 3, -1, 5]], dtype=torch.int32), torch.ones(1, 6), 2, pl)
    assert none.send_counts == [0, 1] and none.meta_expert.tolist() == [[-1, -1, 0, 1, -1, 2]]


@pytest.mark.parametrize("world,kind", [(2, "contiguous"), (2, "balanced"), (4, "balanced")])
def test_ep_forward_gloo_ranks(tmp_path, world, kind):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), kind), nprocs=world, join=True)
    got = np.concatenate([np.load(tmp_path / f"rank{r}.npy") for r in range(world)])
    o, cfg, w, x = _setup()
    r = o.route_fp32(x, w.router, None, K)
    ref = o.moe_layer_fp64(cfg, w, x, r.ids, r.weights)
    assert np.max(np.abs(got - ref)) <= 2e-2
    assert o.rel_l2(got, ref) <= 1e-2


def test_expert_parallel_module_refuses_bad_placements_and_cpu():
    """Checked on the host before any device work (a one-rank gloo group)."""
    ep = importlib.import_module("unlimited-ocr-max_b200.ep")
    uocr = importlib.import_module("unlimited-ocr-max_b200")
    dist.init_process_group("gloo", rank=0, world_size=1, init_method=f"tcp://127.0.0.1:{_free_port()}")
    try:
        cfg = uocr.MoEConfig()
        bad = [ep.ExpertPlacement([list(range(63))]),                  # an expert missing
               ep.ExpertPlacement([list(range(64)) + [0]]),            # an expert twice
               ep.ExpertPlacement([list(range(32)), list(range(32, 64))])]  # placed for 2 ranks
        for pl in bad:
            with pytest.raises(ValueError, match="placement"):
                ep.ExpertParallelMoE(cfg, device="cpu", placement=pl)
        with pytest.raises(ValueError, match="CUDA"):
            ep.ExpertParallelMoE(cfg, device="cpu")
    finally:
        dist.destroy_process_group()


# ---- failures injected on the host ----------------------------------------------------------------


def _failure_worker(rank: int, world: int, port: int, out_dir: str, mode: str) -> None:
    """mode "absent": rank world-1 never joins the forward (it leaves after a while); the others must
    raise ExchangeError within their timeout. mode "count": rank 1 announces more rows for rank 0
    than it has tokens; every rank must refuse the count table before any row moves."""
    import json
    import time

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = importlib.import_module("unlimited-ocr-max_b200.ep")
    o, cfg, w, x = _setup()
    t_local = T_TOTAL // world
    xl = torch.from_numpy(x[rank * t_local:(rank + 1) * t_local].copy())
    calls = {"rows": 0, "experts": 0}
    real_exchange_rows = ep.exchange_rows

    def counting_exchange_rows(*a, **k):
        calls["rows"] += 1
        return real_exchange_rows(*a, **k)

    ep.exchange_rows = counting_exchange_rows
    if mode == "count" and rank == 1:
        real_plan = ep.plan_dispatch

        def corrupt_plan(*a, **k):
            plan = real_plan(*a, **k)
            plan.send_counts[0] = t_local + 5  # more rows than this rank has tokens
            return plan

        ep.plan_dispatch = corrupt_plan

    def route(xt):
        r = o.route_fp32(xt.numpy(), w.router, None, K)
        return torch.from_numpy(r.ids), torch.from_numpy(r.weights)

    def local_experts(rows, meta_e, meta_w):
        calls["experts"] += 1
        return torch.zeros(rows.shape[0], H)

    def shared(xt, out):
        pass

    result = {"rank": rank}
    if mode == "absent" and rank == world - 1:
        time.sleep(12)  # never takes part; leaves well after the others' timeout
        result["absent"] = True
    else:
        t0 = time.time()
        try:
            ep.ep_forward(xl, route, local_experts, shared, world, E // world, timeout_s=3.0)
            result["raised"] = None
        except ep.ExchangeError as e:
            result["raised"] = str(e)
        result["seconds"] = time.time() - t0
    result.update(calls)
    with open(os.path.join(out_dir, f"fail{rank}.json"), "w") as f:
        json.dump(result, f)
    os._exit(0)  # no destroy_process_group: a peer may be gone


@pytest.mark.parametrize("world", [2, 4])
def test_a_rank_that_never_posts_makes_the_others_raise_in_time(tmp_path, world):
    import json

    mp.spawn(_failure_worker, args=(world, _free_port(), str(tmp_path), "absent"), nprocs=world, join=True)
    for r in range(world - 1):
        res = json.loads((tmp_path / f"fail{r}.json").read_text())
        assert res["raised"] and "not every rank took part within 3 s" in res["raised"], res
        assert res["seconds"] < 10, res
        assert res["rows"] == 0 and res["experts"] == 0, res  # nothing moved after the failed count exchange


def test_a_corrupted_count_is_refused_by_every_rank_before_any_row_moves(tmp_path):
    import json

    world = 2
    mp.spawn(_failure_worker, args=(world, _free_port(), str(tmp_path), "count"), nprocs=world, join=True)
    for r in range(world):
        res = json.loads((tmp_path / f"fail{r}.json").read_text())
        assert res["raised"] and "rank 1 announces" in res["raised"] and "from 24 tokens" in res["raised"], res
        assert res["rows"] == 0 and res["experts"] == 0, res


def test_count_table_checks(tmp_path):
    """The table a healthy step gathers passes; the receive counts are its columns."""
    ep = importlib.import_module("unlimited-ocr-max_b200.ep")
    dist.init_process_group("gloo", rank=0, world_size=1, init_method=f"tcp://127.0.0.1:{_free_port()}")
    try:
        tab = ep.count_table([7], 9, "cpu")
        assert tab.tolist() == [[7, 9]]
        assert ep.exchange_counts([7], "cpu", T=9) == [7]
        with pytest.raises(ep.ExchangeError, match="announces 10 rows for rank 0 from 9 tokens"):
            ep.count_table([10], 9, "cpu")
        with pytest.raises(ep.ExchangeError, match="announces -1 rows"):
            ep.count_table([-1], 9, "cpu")
    finally:
        dist.destroy_process_group()
