"""GPU: the tensor-core dense projection (``uocr_dense_stream``) against the fp64 product and the
reference op's fp32 bits (``dense_bf16_qmv``), on the decoder's projection shapes and ragged ones;
K-blocked and plain weights; repeatability of the split-K reduction."""

from __future__ import annotations

import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def dense():
    return importlib.import_module("unlimited-ocr-max_b200.dense")


@pytest.fixture(scope="module")
def ops():
    return importlib.import_module("unlimited-ocr-max_b200.ops")


def _case(N: int, K: int, M: int, seed: int):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = (torch.randn((N, K), generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    x = torch.randn((M, K), generator=g, device=DEV)
    return w, x


def _kblock(w: torch.Tensor) -> torch.Tensor:
    n, k = w.shape
    return w.reshape(n, k // 16, 16).permute(1, 0, 2).contiguous()


def _close(out: torch.Tensor, w: torch.Tensor, x: torch.Tensor) -> None:
    """Within 1e-4 of sum |w x| of the fp64 product: x enters as two bf16 terms (to 2^-18 of |x|),
    the products accumulate in fp32."""
    ref = x.double() @ w.double().T
    bound = x.double().abs() @ w.double().abs().T
    err = (out.double() - ref).abs()
    assert bool((err <= 1e-4 * bound + 1e-6).all()), float((err / (bound + 1e-30)).max())


# the decoder's projections (attention, dense FFN, lm_head) and ragged shapes
SHAPES = [(1280, 1280), (6848, 1280), (1280, 6848), (300, 272), (16, 16), (200, 4096)]


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("M", [1, 3, 8, 13])
def test_dense_projection_matches_fp64(dense, N, K, M):
    w, x = _case(N, K, M, 7 * N + K + M)
    p = dense.DenseProjection(K, N, kblocked=True).load_state_dict({"weight": _kblock(w)})
    out = p.decode_rows(x)
    _close(out, w, x)
    p.check_status()


def test_lm_head_shape(dense):
    N, K = 129280, 1280
    w, x = _case(N, K, 8, 11)
    p = dense.DenseProjection(K, N, kblocked=False).load_state_dict({"weight": w})
    out = p.decode_rows(x)
    _close(out, w, x)
    p.check_status()


@pytest.mark.parametrize("N,K", [(1280, 1280), (1280, 6848), (300, 272)])
def test_kblocked_and_plain_and_repeat_give_the_same_bits(dense, N, K):
    w, x = _case(N, K, 8, 3)
    a = dense.DenseProjection(K, N, kblocked=True).load_state_dict({"weight": _kblock(w)})
    b = dense.DenseProjection(K, N, kblocked=False).load_state_dict({"weight": w})
    first = a.decode_rows(x)
    assert torch.equal(first, b.decode_rows(x))
    for _ in range(3):  # split-K counters are restored by every call
        assert torch.equal(first, a.decode_rows(x))
    a.check_status()


@pytest.mark.parametrize("N,K", [(1280, 1280), (6848, 1280)])
def test_agrees_with_the_reference_op(dense, ops, N, K):
    """The reference op's fp32 result (``dense_bf16_qmv``, the reference's operation order) and the
    tensor-core stream agree to the products' accumulation order."""
    w, x = _case(N, K, 8, 5)
    ref_op = ops.dense_bf16_qmv(x, _kblock(w))
    out = dense.DenseProjection(K, N).load_state_dict({"weight": _kblock(w)}).decode_rows(x)
    bound = x.double().abs() @ w.double().abs().T
    assert bool(((out.double() - ref_op.double()).abs() <= 2e-4 * bound + 1e-6).all())


def test_rows_are_independent_of_the_batch(dense):
    w, x = _case(1280, 1280, 8, 9)
    p = dense.DenseProjection(1280, 1280).load_state_dict({"weight": _kblock(w)})
    full = p.decode_rows(x)
    for m in range(8):
        assert torch.equal(p.decode_rows(x[m:m + 1]), full[m:m + 1])


def test_refusals(dense):
    with pytest.raises(ValueError, match="multiple of 16"):
        dense.DenseProjection(100, 64)
    p = dense.DenseProjection(256, 64)
    with pytest.raises(ValueError, match="declared"):
        p.load_state_dict({"weight": torch.zeros(64, 256, dtype=torch.bfloat16, device=DEV)})
    p.load_state_dict({"weight": torch.zeros(16, 64, 16, dtype=torch.bfloat16, device=DEV)})
    with pytest.raises(ValueError, match="fp32"):
        p.decode_rows(torch.zeros(2, 128, device=DEV))
    assert p.decode_rows(torch.zeros(0, 256, device=DEV)).shape == (0, 64)


@pytest.mark.parametrize("parts,K", [((1280, 1280, 1280), 1280), ((6848, 6848), 1280), ((200, 72, 1000), 272)])
def test_fused_projection_parts_match_fp64(dense, parts, K):
    ws, xs = zip(*[_case(n, K, 8, 31 + i) for i, n in enumerate(parts)])
    x = xs[0]
    f = dense.FusedProjection(K, parts).load_weights([_kblock(w) for w in ws])
    outs = f.decode_rows(x)
    assert len(outs) == len(parts)
    for o, w in zip(outs, ws):
        _close(o, w, x)
    f.check_status()
