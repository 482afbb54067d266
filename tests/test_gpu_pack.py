"""The packed weight blocks (uocr_moe_pack_w13 / _w2 / _shared) byte for byte against a numpy
statement of the layout: every row followed by 16 zero bytes; w13 blocks of P row pairs
[gate P rows | up P rows | int8: gate scales | up scales] (P = 8 bf16, 16 int8); w2 blocks of
32 rows [rows | int8: scales]."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


PAD = 16


def padded(rows: np.ndarray) -> bytes:
    return b"".join(r.tobytes() + bytes(PAD) for r in rows)


def w13_ref(gate: np.ndarray, up: np.ndarray, gs, us, P: int) -> bytes:
    E, I, H = gate.shape
    out = bytearray()
    for e in range(E):
        for b in range(I // P):
            rows = slice(b * P, (b + 1) * P)
            out += padded(gate[e, rows]) + padded(up[e, rows])
            if gs is not None:
                out += gs[e, rows].tobytes() + us[e, rows].tobytes()
    return bytes(out)


def w2_ref(down: np.ndarray, ds) -> bytes:
    E, H, I = down.shape
    out = bytearray()
    for e in range(E):
        for b in range(H // 32):
            rows = slice(b * 32, (b + 1) * 32)
            out += padded(down[e, rows])
            if ds is not None:
                out += ds[e, rows].tobytes()
    return bytes(out)


@pytest.mark.parametrize("int8", [False, True])
def test_pack_routed_blocks(uocr, int8):
    L = uocr.load()
    E, I, H, G = 3, 128, 256, 128
    rng = np.random.default_rng(3)
    if int8:
        gate, up = (rng.integers(-127, 128, (E, I, H), dtype=np.int8) for _ in range(2))
        down = rng.integers(-127, 128, (E, H, I), dtype=np.int8)
        gs, us = (rng.random((E, I, H // G), dtype=np.float32) for _ in range(2))
        ds = rng.random((E, H, I // G), dtype=np.float32)
    else:
        gate, up = (rng.integers(0, 1 << 16, (E, I, H), dtype=np.uint16) for _ in range(2))
        down = rng.integers(0, 1 << 16, (E, H, I), dtype=np.uint16)
        gs = us = ds = None
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    tg, tu, td = dev(gate.view(np.int16) if not int8 else gate), dev(up.view(np.int16) if not int8 else up), \
        dev(down.view(np.int16) if not int8 else down)
    tgs, tus, tds = (dev(a) if a is not None else None for a in (gs, us, ds))
    n13, n2 = L.uocr_moe_w13_bytes(E, I, H, G, int(int8)), L.uocr_moe_w2_bytes(E, H, I, G, int(int8))
    o13 = torch.zeros(n13, dtype=torch.uint8, device=DEV)
    o2 = torch.zeros(n2, dtype=torch.uint8, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    assert L.uocr_moe_pack_w13(tg.data_ptr(), tu.data_ptr(), ptr(tgs), ptr(tus), E, I, H, G, int(int8),
                               o13.data_ptr(), st) == 0, L.uocr_last_error()
    assert L.uocr_moe_pack_w2(td.data_ptr(), ptr(tds), E, H, I, G, int(int8), o2.data_ptr(), st) == 0
    torch.cuda.synchronize()
    P = 16 if int8 else 8
    assert o13.cpu().numpy().tobytes() == w13_ref(gate, up, gs, us, P)
    assert o2.cpu().numpy().tobytes() == w2_ref(down, ds)


def test_pack_shared_blocks(uocr):
    L = uocr.load()
    S, I, H = 2, 128, 256
    rng = np.random.default_rng(4)
    gate, up = (rng.integers(0, 1 << 16, (S * I, H), dtype=np.uint16) for _ in range(2))
    down = rng.integers(0, 1 << 16, (H, S * I), dtype=np.uint16)
    dev = lambda a: torch.from_numpy(a.view(np.int16)).to(DEV)  # noqa: E731
    o13 = torch.zeros(L.uocr_moe_w13_bytes(S, I, H, 128, 0), dtype=torch.uint8, device=DEV)
    o2 = torch.zeros(L.uocr_moe_w2_bytes(S, H, I, 128, 0), dtype=torch.uint8, device=DEV)
    assert L.uocr_moe_pack_shared(dev(gate).data_ptr(), dev(up).data_ptr(), dev(down).data_ptr(), S, I, H,
                                  o13.data_ptr(), o2.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert o13.cpu().numpy().tobytes() == w13_ref(gate.reshape(S, I, H), up.reshape(S, I, H), None, None, 8)
    want2 = np.stack([down[:, q * I:(q + 1) * I] for q in range(S)])
    assert o2.cpu().numpy().tobytes() == padded(want2.reshape(S * H, I))
