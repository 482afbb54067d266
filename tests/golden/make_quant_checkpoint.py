"""Golden files for the int8 checkpoint quantiser: a small synthetic bf16 model file and the int8
file the reference's own tool writes from it.

    python tests/golden/make_quant_checkpoint.py <reference checkout>

writes ``quant_ckpt_in.safetensors`` (routed experts of two decoder layers plus tensors that must
pass through untouched, among them names that nearly match the expert pattern) and
``quant_ckpt_out.safetensors``, made by running ``quantize_file`` of
``tools/quantize_int8.py`` (imported as a module; numpy and the standard library only) on it.
The weights hold the quantiser's edge cases: an all-zero group, rint ties at .5 in both
directions, an amax set by a negative element, and bf16 subnormals.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))


def bf16(a: np.ndarray) -> torch.Tensor:
    """fp32 values rounded to bf16 (round to nearest even)."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def weights(rng: np.random.Generator) -> dict[str, torch.Tensor]:
    t: dict[str, torch.Tensor] = {}
    for layer in (1, 2):
        for e in (0, 1):
            for proj, (n, k) in (("gate_proj", (8, 256)), ("up_proj", (8, 256)), ("down_proj", (16, 128))):
                w = rng.standard_normal((n, k)).astype(np.float32) * np.float32(0.02)
                if (layer, e, proj) == (1, 0, "gate_proj"):
                    w[0, :128] = 0.0                                   # all-zero group: scale 1.0, q 0
                    w[1, 128:] = 0.0                                   # amax 127 -> scale 1.0: ties
                    w[1, 128:137] = [127.0, 2.5, 3.5, -2.5, -0.5, 0.5, 1.5, -1.5, 126.5]
                    w[2, :128] = rng.standard_normal(128).astype(np.float32) * np.float32(3e-39)  # subnormals
                    w[3, :128] = rng.uniform(-0.1, 0.1, 128).astype(np.float32)
                    w[3, 17] = -0.5                                    # amax from the minimum
                t[f"model.layers.{layer}.mlp.experts.{e}.{proj}.weight"] = bf16(w)
    t["model.embed_tokens.weight"] = torch.from_numpy(rng.standard_normal((4, 8)).astype(np.float32))
    t["model.layers.1.mlp.gate.weight"] = bf16(rng.standard_normal((2, 256)) * 0.02)
    t["model.layers.1.mlp.shared_experts.gate_proj.weight"] = bf16(rng.standard_normal((8, 256)) * 0.02)
    t["model.layers.1.mlp.experts.0.gate_proj.bias"] = bf16(rng.standard_normal(8) * 0.02)
    t["model.norm.weight"] = bf16(np.ones(256))
    return t


def main(ref_root: Path) -> None:
    ck = __import__("importlib").import_module("unlimited-ocr-max_b200.checkpoint")
    spec = importlib.util.spec_from_file_location("ref_quantize_int8", ref_root / "tools" / "quantize_int8.py")
    quant = importlib.util.module_from_spec(spec)
    sys.modules["ref_quantize_int8"] = quant
    spec.loader.exec_module(quant)

    src, dst = HERE / "quant_ckpt_in.safetensors", HERE / "quant_ckpt_out.safetensors"
    ck.write_safetensors(src, weights(np.random.default_rng(2024)), {"format": "pt"})
    report = quant.quantize_file(src, dst, expect_sha=None, progress_every=0)
    print(report["source_sha256"], dst.stat().st_size)


if __name__ == "__main__":
    main(Path(sys.argv[1]))
