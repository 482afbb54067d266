"""The C ABI boundary on any host: the library loads, exports every entry point the header
declares, and the host-side checks refuse bad calls with the reference ops' messages before
anything reaches a device. No compute call is made here."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "uocr_moe.h"


def header_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(uocr_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_reference_ops():
    names = header_functions()
    for op in ("uocr_moe_bf16_qmv", "uocr_moe_int8_qmv", "uocr_int8_dequant_expert", "uocr_dense_bf16_qmv",
               "uocr_moe_route", "uocr_moe_decode"):
        assert op in names


def test_library_exports_every_declared_symbol(uocr):
    lib = uocr.load()
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, missing
    from importlib import import_module

    sigs = import_module("unlimited-ocr-max_b200._lib").SIGNATURES
    assert sorted(sigs) == header_functions()
    assert lib.uocr_abi_version() == 6


def test_only_the_c_abi_is_exported(uocr):
    """-fvisibility=hidden: the kernels and helpers are not part of the ABI."""
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(uocr.LIB_PATH)], capture_output=True, text=True).stdout
    ours = sorted({line.split()[-1] for line in out.splitlines() if " T " in line and "uocr" in line})
    assert ours == header_functions()


def _null_call(lib, name, *args):
    fn = getattr(lib, name)
    return fn(*args), lib.uocr_last_error().decode()


@pytest.mark.parametrize(
    "dims,message",
    [
        ((6, 8, 5, 32, 6, 5, 8, 32), "moe_bf16_qmv: x and output disagree on k"),
        ((6, 8, 6, 32, 5, 5, 8, 32), "moe_bf16_qmv: expert_ids and output disagree on k"),
        ((6, 8, 6, 32, 6, 5, 9, 32), "moe_bf16_qmv: w and output disagree on N"),
        ((6, 8, 6, 24, 6, 5, 8, 32), "moe_bf16_qmv: w and x disagree on K"),
        ((6, 8, 6, 32, 6, 0, 8, 32), "moe_bf16_qmv: the expert stack is empty"),
    ],
)
def test_bf16_qmv_shape_errors(uocr, dims, message):
    """kernels/moe_bf16.mojo:276-285, checked before any launch (null device pointers are fine)."""
    out_r, out_c, x_r, x_c, ids_l, w_e, w_n, w_k = dims
    rc, err = _null_call(uocr.load(), "uocr_moe_bf16_qmv", None, out_r, out_c, None, x_r, x_c, None, ids_l, None,
                         w_e, w_n, w_k, None)
    assert rc == 1 and err == message


def test_int8_qmv_group_miscount(uocr):
    rc, err = _null_call(uocr.load(), "uocr_moe_int8_qmv", None, 2, 4, None, 2, 32, None, 2, None, 3, 4, 32, None,
                         3, 4, 5, None)
    assert rc == 1 and err == "moe_int8_qmv: K must be a multiple of the group count"


def test_dequant_checks(uocr):
    lib = uocr.load()
    rc, err = _null_call(lib, "uocr_int8_dequant_expert", None, 4, 32, None, 3, 4, 32, None, 3, 4, 5, None, 1, None)
    assert rc == 1 and err == "int8_dequant_expert: K must be a multiple of the group count"
    rc, err = _null_call(lib, "uocr_int8_dequant_expert", None, 4, 32, None, 3, 4, 32, None, 3, 4, 4, None, 2, None)
    assert rc == 1 and err == "int8_dequant_expert: `expert_idx` must be a single int32"


def test_dense_checks(uocr):
    lib = uocr.load()
    rc, err = _null_call(lib, "uocr_dense_bf16_qmv", None, 2, 8, None, 2, 32, None, 2, 8, 8, 1, None)
    assert rc == 1 and err == "dense_bf16_qmv: w is not K-blocked by KBLOCK"
    rc, err = _null_call(lib, "uocr_dense_bf16_qmv", None, 2, 8, None, 2, 48, None, 2, 8, 16, 1, None)
    assert rc == 1 and err == "dense_bf16_qmv: w and x disagree on K"


def test_zero_rows_launch_nothing(uocr):
    """k = 0 returns OK without touching the device (a warm-up launch can have no rows)."""
    rc, _ = _null_call(uocr.load(), "uocr_moe_bf16_qmv", None, 0, 8, None, 0, 32, None, 0, None, 5, 8, 32, None)
    assert rc == 0


def test_decode_rejects_bad_layers(uocr):
    lib = uocr.load()
    L = uocr._lib.UocrMoeLayer()
    L.hidden, L.inter, L.n_routed, L.n_shared, L.top_k, L.group = 1280, 896, 64, 2, 6, 128
    rc = lib.uocr_moe_decode(ctypes.byref(L), None, 1, None, None, None, None, None, 0, None)
    assert rc == 1 and "null weight pointer" in lib.uocr_last_error().decode()
    L.inter = 900
    rc = lib.uocr_moe_decode(ctypes.byref(L), None, 1, None, None, None, None, None, 0, None)
    assert rc == 1 and "multiple of 128" in lib.uocr_last_error().decode()
    assert lib.uocr_moe_decode_workspace_bytes(ctypes.byref(L), 8) > 0


def test_ops_refuse_cpu_tensors(uocr):
    """No CPU fallback: host tensors are an error, not a slow path."""
    x = torch.zeros(2, 32)
    ids = torch.zeros(2, dtype=torch.int32)
    w = torch.zeros(3, 4, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA tensor"):
        uocr.ops.moe_bf16_qmv(x, ids, w)
    with pytest.raises(ValueError, match="CUDA device only"):
        uocr.UocrMoE(uocr.MoEConfig(), device="cpu")


def test_config_validation(uocr):
    C = uocr.MoEConfig
    with pytest.raises(uocr.ConfigError, match="renormalisation"):
        C(norm_topk_prob=True)
    with pytest.raises(uocr.ConfigError, match="scoring_func"):
        C(scoring_func="sigmoid")
    with pytest.raises(uocr.ConfigError, match="group size"):
        C(hidden_size=1216, int8_experts=True)
    assert C().shared_experts_dim == 1792


def test_packed_sizes_and_refusals(uocr):
    """Packed item sizes follow the layout; bad packing calls are refused on the host."""
    L = uocr.load()
    # items: atoms of 128 rows x 128 bytes (+ int8 scales, one fp32 per row and atom); gate|up
    # row blocks of 64 pairs with 2 atoms per item, down row blocks of 128 rows (int8: 1 atom)
    atom = 128 * 128
    assert L.uocr_moe_w13_bytes(64, 896, 1280, 128, 1) == 64 * 14 * 5 * (2 * atom + 2 * 128 * 4)
    assert L.uocr_moe_w13_bytes(64, 896, 1280, 128, 0) == 64 * 14 * 10 * 2 * atom
    assert L.uocr_moe_w2_bytes(64, 1280, 896, 128, 1) == 64 * 10 * 7 * (atom + 128 * 4)
    assert L.uocr_moe_w2_bytes(64, 1280, 896, 128, 0) == 64 * 10 * 7 * 2 * atom
    assert L.uocr_moe_w13_bytes(64, 896, 1280, 128, 0) == 64 * 2 * 896 * 1280 * 2  # bf16: no padding
    assert L.uocr_moe_w13_bytes(64, 896, 1152, 128, 1) == 0  # int8 gate|up needs H % 256
    assert L.uocr_moe_w13_bytes(64, 896, 1280, 64, 1) == 0  # only the checkpoint's G = 128
    rc = L.uocr_moe_pack_w13(None, None, None, None, 4, 100, 256, 128, 0, None, None)
    assert rc == 1 and b"pack_w13" in L.uocr_last_error()
    rc = L.uocr_moe_pack_w2(None, None, 4, 256, 896, 64, 1, None, None)
    assert rc == 4 and b"group size" in L.uocr_last_error()


def test_ep_dispatch_combine_refusals(uocr):
    """Argument checks of the expert-parallel bookkeeping entry points (no device work)."""
    lib = uocr.load()
    err = lambda: lib.uocr_last_error().decode()  # noqa: E731
    assert lib.uocr_moe_ep_dispatch_workspace_bytes(16384, 4) > 16384
    assert lib.uocr_moe_ep_dispatch_workspace_bytes(16, 9) == 0
    args = [None, 16, 1280, None, None, 6, None, None, 64]
    assert lib.uocr_moe_ep_dispatch(*args, 9, None, None, None, None, None, 0, None) == 4 and "world=9" in err()
    assert lib.uocr_moe_ep_dispatch(None, 16, 1284, None, None, 6, None, None, 64, 2, None, None, None, None, None, 0,
                                    None) == 1 and "multiple of 8" in err()
    assert lib.uocr_moe_ep_dispatch(*args, 2, None, None, None, None, None, 0, None) == 1 and "null" in err()
    assert lib.uocr_moe_ep_combine(None, 4, None, 16, 0, 1280, None, None, None) == 4 and "world=0" in err()
    assert lib.uocr_moe_ep_combine(None, 4, None, 16, 2, 1280, None, None, None) == 1 and "null" in err()
    assert lib.uocr_moe_ep_combine(None, 0, None, 0, 2, 1280, None, None, None) == 0


def test_widening_entry_points_refuse_before_any_launch(uocr):
    """The quantiser, dense stream, norm, n-gram guard and paged attention check their arguments on
    the host (null device pointers are fine: nothing is launched)."""
    lib = uocr.load()
    rc, err = _null_call(lib, "uocr_quantize_int8_g128", None, 1, 4, 200, None, None, None, None)
    assert rc == 1 and err == "K=200 is not divisible by the group size 128"
    rc, err = _null_call(lib, "uocr_quantize_int8_g128", None, 7, 4, 256, None, None, None, None)
    assert rc == 1 and "fp32 or bf16" in err
    assert _null_call(lib, "uocr_quantize_int8_g128", None, 1, 0, 256, None, None, None, None)[0] == 0  # no rows

    assert lib.uocr_dense_packed_bytes(1280, 1280) == 10 * 10 * 32768
    assert lib.uocr_dense_packed_bytes(300, 272) == 3 * 3 * 32768  # rows and K padded to 128
    assert lib.uocr_dense_packed_bytes(16, 20) == 0  # K not a multiple of 16
    rc, err = _null_call(lib, "uocr_dense_pack", None, 1, 64, 100, None, None)
    assert rc == 1 and "multiple of 16" in err
    rc, err = _null_call(lib, "uocr_dense_stream", None, 64, 256, None, 2, None, None, 0, None)
    assert rc == 1 and err == "dense_stream: null pointer"
    assert _null_call(lib, "uocr_dense_stream", None, 64, 256, None, 0, None, None, 0, None)[0] == 0  # M = 0

    rc, err = _null_call(lib, "uocr_residual_rmsnorm", None, None, None, 2, 0, ctypes.c_float(1e-6), None, None)
    assert rc == 1 and "bad shape" in err
    rc, err = _null_call(lib, "uocr_residual_rmsnorm", None, None, None, 2, 8, ctypes.c_float(-1.0), None, None)
    assert rc == 1 and "eps" in err

    rc, err = _null_call(lib, "uocr_ngram_block", None, 2, 100, None, 0, None, None, None)
    assert rc == 1 and err == "ngram_block: history is empty"
    rc, err = _null_call(lib, "uocr_ngram_block", None, 2, 100, None, 8, None, None, None)
    assert rc == 1 and err == "ngram_block: `ngram` must be a single int32"

    assert lib.uocr_paged_attention_workspace_bytes(8, 10, 5) > 8192
    assert lib.uocr_paged_attention_workspace_bytes(8, 13, 5) == 0
    rc, err = _null_call(lib, "uocr_paged_decode_attention", None, None, None, 8, 10, 64, None, 4, 2, 0, None, 5,
                         None, None, ctypes.c_float(0.1), None, None, 0, None)
    assert rc == 4 and "head_dim" in err
    rc, err = _null_call(lib, "uocr_paged_decode_attention", None, None, None, 8, 10, 128, None, 4, 2, 2, None, 5,
                         None, None, ctypes.c_float(0.1), None, None, 0, None)
    assert rc == 1 and "bad pool" in err
