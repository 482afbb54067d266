"""GPU: the benchmark's 11-layer decode stack, built and captured in one CUDA graph exactly as
``bench.py`` does it (``build_stack`` + ``time_stack``: distinct seeded layers, every layer's
input and output a slice of one [L, B, H] buffer), checked layer by layer against the oracle.

Per layer: the routing ids and weights are bit-exact with the oracle's fp32 gate, and the output
is within the reference's float64 bar (cosine >= 0.99999, rel <= 1e-4) and the north-star bar
(max-abs <= 2e-2, rel-L2 <= 1e-2) of the float64 layer fed the same routing.
"""

from __future__ import annotations

import importlib
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from test_oracle import weights_from_state

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_for_stack_test", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    return bench


@pytest.mark.parametrize("int8,B", [(True, 8), (False, 8), (True, 1)])
def test_graph_captured_stack_matches_the_oracle_layer_by_layer(uocr, oracle, int8, B):
    bench = _bench()
    synth = importlib.import_module("unlimited-ocr-max_b200.synth")
    dev = torch.device("cuda", 0)
    L, seed0 = 11, 1000 + 7 * B + int(int8)
    mods, xs, outs, ids, wts = bench.build_stack(uocr, synth, int8, L, B, dev, seed0)
    g, ms, _ = bench.time_stack(torch, mods, xs, outs, ids, wts, 3, 3, None)
    assert ms > 0
    torch.cuda.synchronize()
    for m in mods:
        m.check_status()
    cfg = oracle.MoEConfig()
    for l in range(L):
        # the layer's weights exactly as build_stack drew them (same seed, same device generator)
        state = {k: v.cpu() for k, v in synth.layer_state(uocr.MoEConfig(int8_experts=int8), seed0 + l,
                                                          device=dev).items()}
        w = weights_from_state(oracle, state, int8)
        x = xs[l].cpu().numpy()
        r = oracle.route_fp32(x, w.router, None, 6)
        assert np.array_equal(ids[l].cpu().numpy(), r.ids), l
        assert np.array_equal(wts[l].cpu().numpy().view(np.uint32), r.weights.view(np.uint32)), l
        got = outs[l].cpu().numpy()
        ref = oracle.moe_layer_fp64(cfg, w, x, r.ids, r.weights)
        for i in range(B):
            assert oracle.cosine(got[i], ref[i]) >= 0.99999, (l, i)
        assert oracle.rel_err(got, ref) <= 1e-4, l
        assert np.max(np.abs(got - ref)) <= 2e-2 and oracle.rel_l2(got, ref) <= 1e-2, l
    del g
