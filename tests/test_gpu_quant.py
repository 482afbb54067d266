"""GPU: the int8 quantiser (``uocr_quantize_int8_g128``) against the reference tool's golden
vectors and the pinned oracle, bit for bit; the checkpoint quantiser against the file the
reference's tool wrote; loading a layer from a safetensors file."""

from __future__ import annotations

import hashlib
import importlib
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def ops():
    return importlib.import_module("unlimited-ocr-max_b200.ops")


@pytest.fixture(scope="module")
def ck():
    return importlib.import_module("unlimited-ocr-max_b200.checkpoint")


def _same(q, s, q_ref, s_ref):
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), np.asarray(s_ref, dtype=np.float32).view(np.uint32))


def _bf16_values(seed: int, n: int, k: int) -> np.ndarray:
    """The golden random case's bf16-valued fp32 weight (tests/golden/make_golden.py)."""
    rng = np.random.default_rng(seed)
    w32 = rng.standard_normal((n, k)).astype(np.float32) * np.float32(0.02)
    bits = w32.view(np.uint32)
    bits = ((bits + np.uint32(0x7FFF) + ((bits >> 16) & np.uint32(1))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    return bits.view(np.float32)


def test_known_answer_tensor(ops):
    g = np.load(GOLDEN / "quantize.npz")
    q, s = ops.quantize_per_group(torch.from_numpy(g["golden_w"]).to(DEV))
    _same(q, s, g["golden_q"], g["golden_scales"])


@pytest.mark.parametrize("case", ["rand0", "rand1", "rand2"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_golden_random_cases(ops, case, dtype):
    g = np.load(GOLDEN / "quantize.npz")
    seed, n, k = (int(v) for v in g[f"{case}_meta"])
    wb = _bf16_values(seed, n, k)
    assert hashlib.sha256(str(wb.dtype).encode() + str(wb.shape).encode() + wb.tobytes()).hexdigest() == str(
        g[f"{case}_w_sha"])
    q, s = ops.quantize_per_group(torch.from_numpy(wb).to(DEV).to(dtype))
    _same(q, s, g[f"{case}_q"], g[f"{case}_scales"])


def _stack(E: int, N: int, K: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(E, N, K, generator=g) * 0.02
    w[0, 0, :128] = 0                                          # all-zero group
    w[0, 1, :128] = torch.randn(128, generator=g) * 3e-39      # subnormal group
    w[0, 2, :128] = 0
    w[0, 2, :9] = torch.tensor([127.0, 2.5, 3.5, -2.5, -0.5, 0.5, 1.5, -1.5, 126.5])  # ties to even
    w[1, 3, 128:256] = -w[1, 3, 128:256].abs()                 # amax from the minimum
    return w.to(torch.bfloat16)


def test_full_layer_stack_equals_the_oracle(ops):
    w = _stack(8, 896, 1280, 5)
    q, s = ops.quantize_per_group(w.to(DEV))
    qr, sr = oracle.quantize_per_group(w.float().numpy())
    _same(q, s, qr, sr)


def test_unaligned_input_takes_the_same_bits(ops):
    w = _stack(2, 64, 384, 6)
    buf = torch.zeros(w.numel() + 1, dtype=torch.bfloat16, device=DEV)
    buf[1:] = w.reshape(-1).to(DEV)
    wu = buf[1:].view(w.shape)                                 # 2 bytes off 16-byte alignment
    q, s = ops.quantize_per_group(wu)
    qr, sr = oracle.quantize_per_group(w.float().numpy())
    _same(q, s, qr, sr)


def test_refusals(ops):
    with pytest.raises(ops.QuantizeError, match="K=200 is not divisible by the group size 128"):
        ops.quantize_per_group(torch.zeros(4, 200, dtype=torch.bfloat16, device=DEV))
    for bad in (float("nan"), float("inf"), -float("inf")):
        w = torch.zeros(4, 256, dtype=torch.bfloat16, device=DEV)
        w[3, 200] = bad
        with pytest.raises(ops.QuantizeError, match="NaN or Inf"):
            ops.quantize_per_group(w)
    q, s = ops.quantize_per_group(torch.zeros(0, 256, dtype=torch.float32, device=DEV))
    assert q.shape == (0, 256) and s.shape == (0, 2)


def test_checkpoint_quantiser_writes_the_reference_tools_file(ck, tmp_path):
    src, ref = GOLDEN / "quant_ckpt_in.safetensors", GOLDEN / "quant_ckpt_out.safetensors"
    out = tmp_path / "int8.safetensors"
    rep = ck.quantize_checkpoint(src, out, tool="quantize_int8.py 1.0")
    assert rep["quantized_tensors"] == 12
    assert out.read_bytes() == ref.read_bytes()
    assert rep["output_sha256"] == hashlib.sha256(ref.read_bytes()).hexdigest()
    # the build's own tool name changes only the metadata
    own = tmp_path / "own.safetensors"
    ck.quantize_checkpoint(src, own)
    with ck.SafetensorsFile(own) as a, ck.SafetensorsFile(ref) as b:
        assert a.metadata["tool"] == ck.TOOL
        assert all(a.raw_bytes(n) == b.raw_bytes(n) for n in b)
