"""The decode entry point that allocates nothing (uocr_moe_decode_noalloc), through the C ABI.

It exists for callers that cannot hand the library a workspace -- hosts whose operator
interface passes only inputs and outputs, or runtimes with all device memory reserved up
front -- and keeps its scratch in a fixed 1 MiB array inside the library. This file is named
to be collected last, so a run that stops at the first failure has already run every other
test; it also passes on its own in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layer(uocr, int8: bool, seed: int):
    synth = __import__("importlib").import_module("unlimited-ocr-max_b200.synth")
    cfg = uocr.MoEConfig(int8_experts=int8)
    return uocr.UocrMoE(cfg, device=DEV).load_state_dict(synth.layer_state(cfg, seed, device=DEV)), synth


@pytest.mark.parametrize("int8", [False, True])
def test_noalloc_matches_the_workspace_entry_point_twice(uocr, oracle, int8):
    lib = uocr.load()
    moe, synth = _layer(uocr, int8, 31 + int(int8))
    stream = torch.cuda.current_stream().cuda_stream
    for call, B in enumerate((8, 3)):  # two calls in a row, the second smaller than the first
        x = synth.hidden_states(B, 1280, 500 + call, device=DEV)
        want = moe.decode_rows(x)
        got = torch.full_like(x, float("nan"))
        rc = lib.uocr_moe_decode_noalloc(ctypes.byref(moe.layer), x.data_ptr(), B, None, got.data_ptr(), stream)
        assert rc == 0, lib.uocr_last_error().decode()
        torch.cuda.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.all(np.isfinite(g))
        # the tolerance the layer tests use, and in fact the same kernels give the same bits
        assert oracle.rel_err(g, w) <= 1e-4
        assert torch.equal(got, want), call


def test_noalloc_refuses_what_does_not_fit(uocr):
    lib = uocr.load()
    assert lib.uocr_moe_decode_noalloc_max_bytes() == 1 << 20
    moe, _ = _layer(uocr, False, 5)
    big = uocr._lib.UocrMoeLayer.from_buffer_copy(moe.layer)
    big.hidden = 64 * 1280  # 8 pairs x (I + H) fp32 no longer fit in 1 MiB
    x = torch.zeros((8, 16), device=DEV)
    rc = lib.uocr_moe_decode_noalloc(ctypes.byref(big), x.data_ptr(), 8, None, x.data_ptr(), None)
    assert rc == 1
    assert "scratch" in lib.uocr_last_error().decode()
    rc = lib.uocr_moe_decode_noalloc(ctypes.byref(moe.layer), x.data_ptr(), 9, None, x.data_ptr(), None)
    assert rc == 1


def test_noalloc_reports_an_expired_wait_and_recovers(uocr):
    """A caller without a workspace still learns of a device-side wait that gave up: the call
    writes NaN over its output, uocr_moe_decode_noalloc_status returns UOCR_EDEVICE once (and
    clears the array's status), and the next call gives the workspace entry point's bits."""
    lib = uocr.load()
    moe, synth = _layer(uocr, True, 41)
    stream = torch.cuda.current_stream().cuda_stream
    x = synth.hidden_states(8, 1280, 600, device=DEV)
    want = moe.decode_rows(x)
    got = torch.zeros_like(x)
    assert lib.uocr_moe_decode_noalloc_status(stream) == 0, lib.uocr_last_error().decode()
    assert lib.uocr_moe_test_wait_extra(1) == 0  # the grid barrier waits for an arrival that never comes
    try:
        rc = lib.uocr_moe_decode_noalloc(ctypes.byref(moe.layer), x.data_ptr(), 8, None, got.data_ptr(), stream)
    finally:
        assert lib.uocr_moe_test_wait_extra(0) == 0
    assert rc == 0
    assert lib.uocr_moe_decode_noalloc_status(stream) == 3
    assert "bounded wait" in lib.uocr_last_error().decode()
    assert torch.isnan(got).all()
    assert lib.uocr_moe_decode_noalloc_status(stream) == 0  # read once: cleared
    rc = lib.uocr_moe_decode_noalloc(ctypes.byref(moe.layer), x.data_ptr(), 8, None, got.data_ptr(), stream)
    assert rc == 0 and lib.uocr_moe_decode_noalloc_status(stream) == 0
    assert torch.equal(got, want)
