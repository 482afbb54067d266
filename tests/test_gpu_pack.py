"""The packed weight items (uocr_moe_pack_w13 / _w2 / _shared) byte for byte against a numpy
statement of the layout: row blocks of 128 rows; an item is `atoms` K ranges of 128 bytes per
row, each a [128 rows][128 B] atom with the 16-byte chunks of row r permuted c -> c ^ (r % 8)
(128-byte swizzle), then for int8 the fp32 scales [atom][row]. gate|up row blocks hold 64 pairs
interleaved by 8 (rows 16i..16i+7 gate, 16i+8..16i+15 up), 2 atoms per item; down row blocks
hold 128 output rows, 1 (int8) or 2 (bf16) atoms per item."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def swizzle(atom: np.ndarray) -> bytes:
    """[R, 128] uint8 -> the 128-byte-swizzled atom."""
    R = atom.shape[0]
    chunks = atom.reshape(R, 8, 16)
    out = np.empty_like(chunks)
    dst = np.arange(8)[None, :] ^ (np.arange(R) % 8)[:, None]
    out[np.arange(R)[:, None], dst] = chunks
    return out.tobytes()


def items(rows: np.ndarray, scales, atoms: int) -> bytes:
    """rows: [128, K] (int8 or uint16) of one row block; scales [128, K/128] fp32 or None."""
    raw = rows.view(np.uint8).reshape(128, -1)
    out = bytearray()
    per_item = atoms * 128
    for i0 in range(0, raw.shape[1], per_item):
        here = min(atoms, (raw.shape[1] - i0) // 128)  # the last item may be shorter
        for a in range(here):
            out += swizzle(np.ascontiguousarray(raw[:, i0 + a * 128:i0 + (a + 1) * 128]))
        if scales is not None:
            g0 = i0 // 128  # int8: one byte per element, so byte offset / 128 = group
            for a in range(here):
                out += np.ascontiguousarray(scales[:, g0 + a]).astype(np.float32).tobytes()
    return bytes(out)


def w13_ref(gate: np.ndarray, up: np.ndarray, gs, us) -> bytes:
    E, I, H = gate.shape
    r = np.arange(128)
    pair = (r >> 4) * 8 + (r & 7)
    is_up = (r & 15) >= 8
    out = bytearray()
    for e in range(E):
        for rb in range(I // 64):
            p = 64 * rb + pair
            rows = np.where(is_up[:, None], up[e, p], gate[e, p])
            sc = None if gs is None else np.where(is_up[:, None], us[e, p], gs[e, p])
            out += items(rows, sc, 2)
    return bytes(out)


def w2_ref(down: np.ndarray, ds) -> bytes:
    E, H, I = down.shape
    out = bytearray()
    for e in range(E):
        for rb in range(H // 128):
            j = slice(128 * rb, 128 * rb + 128)
            out += items(down[e, j], None if ds is None else ds[e, j], 2)
    return bytes(out)


@pytest.mark.parametrize("int8", [False, True])
def test_pack_routed_blocks(uocr, int8):
    L = uocr.load()
    E, I, H, G = 3, 384, 256, 128  # I / 128 = 3: the down rows' last int8 item holds one group
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
    assert o13.cpu().numpy().tobytes() == w13_ref(gate, up, gs, us)
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
    assert o13.cpu().numpy().tobytes() == w13_ref(gate.reshape(S, I, H), up.reshape(S, I, H), None, None)
    want2 = np.stack([down[:, q * I:(q + 1) * I] for q in range(S)])
    assert o2.cpu().numpy().tobytes() == w2_ref(want2, None)
