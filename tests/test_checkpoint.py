"""CPU: the safetensors reader and writer, the int8 quantiser's plan and refusals, and the golden
int8 file (written by the reference's own tool) against the pinned oracle quantiser."""

from __future__ import annotations

import importlib
import io
import json
import struct
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as oracle

ck = importlib.import_module("unlimited-ocr-max_b200.checkpoint")
weights = importlib.import_module("unlimited-ocr-max_b200.weights")
GOLDEN = Path(__file__).resolve().parent / "golden"
SRC, DST = GOLDEN / "quant_ckpt_in.safetensors", GOLDEN / "quant_ckpt_out.safetensors"


def test_golden_int8_file_is_the_oracle_quantiser_of_the_golden_bf16_file():
    with ck.SafetensorsFile(SRC) as fi, ck.SafetensorsFile(DST) as fo:
        assert fo.metadata["scheme"] == ck.SCHEME and fo.metadata["group_size"] == "128"
        assert fo.metadata["format"] == "pt" and fo.metadata["source_sha256"] == ck._sha256(SRC)
        order = sorted(fo.entries, key=lambda n: fo.entries[n]["data_offsets"])
        assert order == sorted(fo.entries)
        quantised = 0
        for name in fi:
            if ck.CHECKPOINT_EXPERT_RE.match(name):
                q, s = oracle.quantize_per_group(fi[name].float().numpy())
                assert np.array_equal(fo[name].numpy(), q), name
                assert np.array_equal(fo[name + "_scales"].numpy().view(np.uint32), s.view(np.uint32)), name
                quantised += 1
            else:
                assert fo.raw_bytes(name) == fi.raw_bytes(name), name
        assert quantised == 12 and len(fo) == len(fi) + 12


def test_golden_files_hold_the_edge_cases():
    with ck.SafetensorsFile(DST) as fo:
        q = fo["model.layers.1.mlp.experts.0.gate_proj.weight"].numpy()
        s = fo["model.layers.1.mlp.experts.0.gate_proj.weight_scales"].numpy()
    assert s[0, 0] == 1.0 and not q[0, :128].any()                      # all-zero group
    assert s[1, 1] == 1.0 and q[1, 128:137].tolist() == [127, 2, 4, -2, 0, 0, 2, -2, 126]  # ties to even
    assert 0 < s[2, 0] < np.finfo(np.float32).tiny                       # subnormal scale
    assert q[3, 17] == -127                                              # amax from the minimum


def test_checkpoint_forms_from_the_header_alone():
    with ck.SafetensorsFile(SRC) as fi, ck.SafetensorsFile(DST) as fo:
        assert weights.is_int8_checkpoint(fi.meta()) is False
        assert weights.is_int8_checkpoint(fo.meta()) is True
        half = fo.meta()
        del half["model.layers.2.mlp.experts.1.up_proj.weight_scales"]
        with pytest.raises(weights.WeightMappingError, match="half-quantized"):
            weights.is_int8_checkpoint(half)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.int8, torch.float16, torch.int64,
                                   torch.uint8, torch.bool])
def test_write_read_round_trip(tmp_path, dtype):
    g = torch.Generator().manual_seed(3)
    t = {
        "b": (torch.randn(3, 5, generator=g) * 100).to(dtype),
        "a": torch.zeros(0, 4, dtype=dtype),
        "c.weight": (torch.randn(7, generator=g) * 100).to(dtype),
    }
    path = tmp_path / "x.safetensors"
    ck.write_safetensors(path, t, {"format": "pt"})
    raw = path.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0 and json.loads(raw[8:8 + n])["__metadata__"] == {"format": "pt"}
    with ck.SafetensorsFile(path) as f:
        assert sorted(f) == sorted(t)
        for k, v in t.items():
            assert f[k].dtype == dtype and torch.equal(f[k], v), k


def _blob(header: dict, data: bytes = b"") -> io.BytesIO:
    h = json.dumps(header).encode()
    return io.BytesIO(struct.pack("<Q", len(h)) + h + data)


@pytest.mark.parametrize("header,msg", [
    ({"x": {"dtype": "Q8", "shape": [1], "data_offsets": [0, 1]}}, "unknown safetensors dtype"),
    ({"x": {"dtype": "F32", "shape": [2], "data_offsets": [0, 4]}}, "needs 8 bytes"),
    ({"x": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}, "bad shape"),
    ({"x": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}, "bad data_offsets"),
    ({"x": {"dtype": "F32", "shape": [1], "data_offsets": [4, 8]}}, "expected 0"),
    ({"__metadata__": [1]}, "__metadata__ is not a JSON object"),
])
def test_header_refusals(header, msg):
    with pytest.raises(ck.SafetensorsError, match=msg):
        ck.read_header(_blob(header, b"\0" * 8))


def test_header_refusals_truncated():
    with pytest.raises(ck.SafetensorsError, match="shorter than 8 bytes"):
        ck.read_header(io.BytesIO(b"\1\0"))
    with pytest.raises(ck.SafetensorsError, match="truncated safetensors header"):
        ck.read_header(io.BytesIO(struct.pack("<Q", 100) + b"{}"))
    with pytest.raises(ck.SafetensorsError, match="implausible"):
        ck.read_header(io.BytesIO(struct.pack("<Q", 0)))


def _entries(**spec) -> dict:
    out, cur = {}, 0
    for name, (dtype, shape) in spec.items():
        n = ck.DTYPES[dtype][0] * int(np.prod(shape))
        out[name.replace("__", ".")] = {"dtype": dtype, "shape": list(shape), "data_offsets": [cur, cur + n]}
        cur += n
    return out


E = "model__layers__1__mlp__experts__0__gate_proj__weight"


@pytest.mark.parametrize("spec,msg", [
    ({E: ("F32", (8, 256))}, "must be BF16, header says F32"),
    ({E: ("BF16", (2, 8, 256))}, "expected a per-expert 2-D"),
    ({E: ("BF16", (8, 200))}, "K=200 is not divisible by the group size 128"),
    ({E: ("I8", (8, 256)), E + "_scales": ("F32", (8, 2))}, "must be BF16, header says I8"),
    ({E: ("BF16", (8, 256)), E + "_scales": ("F32", (8, 2))}, "already carries per-group scales"),
    ({"model__norm__weight": ("BF16", (8,))}, "no expert weights matched"),
])
def test_plan_refusals(spec, msg):
    with pytest.raises(ck.QuantizeError, match=msg):
        ck._plan(_entries(**spec))


def test_plan_selects_by_name_only():
    plan = ck._plan(_entries(**{
        E: ("BF16", (8, 256)),
        "model__layers__1__mlp__shared_experts__gate_proj__weight": ("BF16", (8, 256)),
        "model__layers__1__mlp__experts__0__gate_proj__bias": ("BF16", (8,)),
        "layers__1__mlp__experts__0__gate_proj__weight": ("BF16", (8, 256)),
    }))
    kinds = {name: kind for name, kind, _, _ in plan}
    assert kinds[E.replace("__", ".")] == "quant" and kinds[E.replace("__", ".") + "_scales"] == "scales"
    assert sum(k == "copy" for k in kinds.values()) == 3


def test_pinned_source_sha_is_enforced(tmp_path):
    with pytest.raises(ck.QuantizeError, match="source sha256 mismatch"):
        ck.quantize_checkpoint(SRC, tmp_path / "o.safetensors", expect_sha="0" * 64, device="cpu")
