"""ctypes binding of ``libuocr_moe.so`` (the C ABI declared in ``include/uocr_moe.h``).

There is no fallback: if the library is missing and cannot be built, importing the ops
fails loudly.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libuocr_moe.so"

UOCR_OK, UOCR_EINVAL, UOCR_ECUDA, UOCR_EDEVICE, UOCR_EUNSUPPORTED = 0, 1, 2, 3, 4

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
SZ = ctypes.c_size_t


class UocrEpPeers(ctypes.Structure):
    """Mirror of ``struct uocr_ep_peers`` (include/uocr_moe.h)."""

    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("cap_tokens", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("epoch", ctypes.c_uint64),
        ("buf", ctypes.c_void_p * 8),
    ]


class UocrMoeLayer(ctypes.Structure):
    """Mirror of ``struct uocr_moe_layer`` (include/uocr_moe.h)."""

    _fields_ = [
        ("hidden", ctypes.c_int32),
        ("inter", ctypes.c_int32),
        ("n_routed", ctypes.c_int32),
        ("n_shared", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("group", ctypes.c_int32),
        ("int8", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("router", P),
        ("w13", P),
        ("w2", P),
        ("w13_shared", P),
        ("w2_shared", P),
    ]


#: name -> (restype, argtypes) for every exported entry point
SIGNATURES: dict[str, tuple] = {
    "uocr_last_error": (ctypes.c_char_p, []),
    "uocr_abi_version": (I32, []),
    "uocr_moe_bf16_qmv": (I32, [P, I64, I64, P, I64, I64, P, I64, P, I64, I64, I64, P]),
    "uocr_moe_int8_qmv": (I32, [P, I64, I64, P, I64, I64, P, I64, P, I64, I64, I64, P, I64, I64, I64, P]),
    "uocr_int8_dequant_expert": (I32, [P, I64, I64, P, I64, I64, I64, P, I64, I64, I64, P, I64, P]),
    "uocr_dense_bf16_qmv": (I32, [P, I64, I64, P, I64, I64, P, I64, I64, I64, I32, P]),
    "uocr_quantize_int8_g128": (I32, [P, I32, I64, I64, P, P, P, P]),
    "uocr_residual_rmsnorm": (I32, [P, P, P, I64, I64, ctypes.c_float, P, P]),
    "uocr_ngram_block": (I32, [P, I64, I64, P, I64, P, P, P]),
    "uocr_rope_qkv": (I32, [P, I64, I64, I64, P, P, P, P, P, P]),
    "uocr_embed_rows": (I32, [P, I64, I64, P, I64, P, P]),
    "uocr_silu_mul": (I32, [P, I64, I64, P, P]),
    "uocr_paged_attention_workspace_bytes": (SZ, [I64, I64, I64]),
    "uocr_paged_decode_attention": (I32, [P, P, P, I64, I64, I64, P, I64, I64, I64, P, I64, P, P, ctypes.c_float, P, P,
                                          SZ, P]),
    "uocr_dense_packed_bytes": (SZ, [I64, I64]),
    "uocr_dense_pack": (I32, [P, I32, I64, I64, P, P]),
    "uocr_dense_stream_workspace_bytes": (SZ, [I64, I64]),
    "uocr_dense_stream": (I32, [P, I64, I64, P, I64, P, P, SZ, P]),
    "uocr_moe_w13_bytes": (SZ, [I64, I64, I64, I64, I32]),
    "uocr_moe_w2_bytes": (SZ, [I64, I64, I64, I64, I32]),
    "uocr_moe_pack_w13": (I32, [P, P, P, P, I64, I64, I64, I64, I32, P, P]),
    "uocr_moe_pack_w2": (I32, [P, P, I64, I64, I64, I64, I32, P, P]),
    "uocr_moe_pack_shared": (I32, [P, P, P, I64, I64, I64, P, P, P]),
    "uocr_moe_route": (I32, [P, I64, I64, P, I64, P, I64, P, P, P]),
    "uocr_moe_decode_workspace_bytes": (SZ, [ctypes.POINTER(UocrMoeLayer), I64]),
    "uocr_moe_decode": (I32, [ctypes.POINTER(UocrMoeLayer), P, I64, P, P, P, P, P, SZ, P]),
    "uocr_moe_prefill_workspace_bytes": (SZ, [ctypes.POINTER(UocrMoeLayer), I64]),
    "uocr_moe_prefill": (I32, [ctypes.POINTER(UocrMoeLayer), P, I64, P, P, P, P, P, SZ, P]),
    "uocr_moe_ep_experts_workspace_bytes": (SZ, [ctypes.POINTER(UocrMoeLayer), I64]),
    "uocr_moe_ep_experts": (I32, [ctypes.POINTER(UocrMoeLayer), P, I64, P, P, P, P, SZ, P]),
    "uocr_moe_shared_workspace_bytes": (SZ, [ctypes.POINTER(UocrMoeLayer), I64]),
    "uocr_moe_shared_forward": (I32, [ctypes.POINTER(UocrMoeLayer), P, I64, P, I32, P, SZ, P]),
    "uocr_moe_ep_dispatch_workspace_bytes": (SZ, [I64, I64]),
    "uocr_moe_ep_dispatch": (I32, [P, I64, I64, P, P, I64, P, P, I64, I64, P, P, P, P, P, SZ, P]),
    "uocr_moe_ep_combine": (I32, [P, I64, P, I64, I64, I64, P, P, P]),
    "uocr_moe_device_status": (I32, [P, P]),
    "uocr_moe_decode_set_trace": (I32, [P, SZ]),
    "uocr_moe_decode_noalloc_max_bytes": (SZ, []),
    "uocr_moe_decode_noalloc": (I32, [ctypes.POINTER(UocrMoeLayer), P, I64, P, P, P]),
    "uocr_moe_decode_noalloc_status": (I32, [P]),
    "uocr_moe_ep_peer_buffer_bytes": (SZ, [I64, I64, I64, I64]),
    "uocr_moe_ep_peer_workspace_bytes": (SZ, [ctypes.POINTER(UocrMoeLayer), ctypes.POINTER(UocrEpPeers)]),
    "uocr_moe_ep_peer_dispatch": (I32, [ctypes.POINTER(UocrEpPeers), P, I64, P, P, P, P, I64, P, P, SZ, P]),
    "uocr_moe_ep_peer_experts": (I32, [ctypes.POINTER(UocrMoeLayer), ctypes.POINTER(UocrEpPeers), P, SZ, P]),
    "uocr_moe_ep_peer_combine": (I32, [ctypes.POINTER(UocrEpPeers), P, I64, P, P, P]),
    "uocr_ipc_export": (I32, [P, P, ctypes.POINTER(ctypes.c_uint64)]),
    "uocr_ipc_import": (I32, [P, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]),
    "uocr_ipc_close": (I32, [P, ctypes.c_uint64]),
    "uocr_moe_test_wait_extra": (I32, [I32]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load (building first if absent) ``libuocr_moe.so`` and declare its signatures."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                from . import build as _build

                _build.build()
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class UocrError(RuntimeError):
    """A libuocr_moe call failed (status code + message)."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def check(code: int) -> None:
    """Raise the reference's error kinds: shape errors as ValueError with the op's message."""
    if code == UOCR_OK:
        return
    msg = load().uocr_last_error().decode()
    if code == UOCR_EINVAL:
        raise ValueError(msg)
    raise UocrError(code, msg)
