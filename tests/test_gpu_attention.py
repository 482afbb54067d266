"""GPU: paged decode attention (``uocr_paged_decode_attention``) against the float64 restatement of
paged_decode_attention (decoder.py:425-437) over the reference's page-pool layout: the new rows
stored bit for bit at their write index (and nothing else of the pool touched), the attention
within 2e-5 of float64, ragged lengths, a ring overwrite inside the attended rows, another layer
of the pool, B = 8 at the model's shape (10 heads x 128, 512 + 128 rows), repeat bit-equality."""

from __future__ import annotations

import importlib
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    return importlib.import_module("unlimited-ocr-max_b200.ops")


def _case(B, heads, layers, cols, attend, write, seed):
    rng = np.random.default_rng(seed)
    pages = B * cols + 1  # the last page is the null page
    pool = rng.standard_normal((pages, 2, layers, 128, heads, 128)).astype(np.float32)
    lut = np.full((B, cols), pages - 1, dtype=np.int32)
    perm = rng.permutation(B * cols)
    for b in range(B):
        lut[b] = perm[b * cols:(b + 1) * cols]
    q, k, v = (rng.standard_normal((B, heads, 128)).astype(np.float32) for _ in range(3))
    return pool, lut, q, k, v, np.asarray(write, np.int32), np.asarray(attend, np.int32)


def _run(ops, pool, lut, q, k, v, write, attend, layer, scale):
    t = lambda a: torch.from_numpy(a).to(DEV)  # noqa: E731
    tp = t(pool)
    out = ops.paged_decode_attention(t(q), t(k), t(v), tp, layer, t(lut), t(write), t(attend), scale)
    return out.cpu().numpy(), tp.cpu().numpy()


@pytest.mark.parametrize("B,heads,layers,cols,attend,write,layer", [
    (4, 10, 3, 5, [1, 37, 300, 640], [0, 36, 299, 200], 1),   # ragged; row 3 overwrites a ring slot
    (8, 10, 2, 5, [640] * 8, [512, 520, 600, 639, 513, 530, 577, 600], 0),  # the model's decode shape
    (3, 4, 1, 2, [129, 16, 17], [128, 15, 3], 0),
])
def test_matches_float64_and_stores_exactly(ops, oracle, B, heads, layers, cols, attend, write, layer):
    pool, lut, q, k, v, wi, al = _case(B, heads, layers, cols, attend, write, 100 + B)
    scale = 1.0 / math.sqrt(128)
    got, pool_after = _run(ops, pool, lut, q, k, v, wi, al, layer, scale)
    ref, pool_ref = oracle.paged_decode_attention_ref(q, k, v, pool, layer, lut, wi, al, scale)
    assert np.array_equal(pool_after.view(np.uint32), pool_ref.view(np.uint32))
    assert np.max(np.abs(got - ref)) <= 2e-5, float(np.max(np.abs(got - ref)))
    again, _ = _run(ops, pool, lut, q, k, v, wi, al, layer, scale)
    assert np.array_equal(again.view(np.uint32), got.view(np.uint32))


def test_one_row_attends_only_itself(ops):
    """attend_len 1: the output is the new v row itself (softmax over one score)."""
    pool, lut, q, k, v, wi, al = _case(2, 10, 1, 1, [1, 1], [0, 0], 7)
    got, _ = _run(ops, pool, lut, q, k, v, wi, al, 0, 0.125)
    assert np.allclose(got, v, rtol=0, atol=1e-6)
