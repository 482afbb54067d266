"""GPU: the no-repeat-n-gram guard (``uocr_ngram_block``) against the oracle restatement of the
reference's processor, as the reference's own kernel tests check it (tests/test_kernels_ngram.py):
the kernel gets only each sequence's last ``window`` ids, must ban exactly the oracle's set (to
-3.0e38) and return every other logit bit for bit; one row and B rows; n = 1, 3, 35; n < 1 and
short histories pass through; rows do not mix; the checkpoint's vocabulary at B = 8; in place."""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
WINDOW = 128  # the R-SWA ring, the guard's window in the reference
VOCAB = 4096
REAL_VOCAB = 129280


@pytest.fixture(scope="module")
def ng():
    return importlib.import_module("unlimited-ocr-max_b200.ngram")


def _sequences(vocab: int, seed: int) -> list[list[int]]:
    """Four sequences longer than the window that the guard treats differently: a 40-id motif
    repeated inside the window (bans), distinct ids only (no ban at n >= 2), period 10 (bans), and
    the motif's first occurrence outside the window (no ban at n >= 2)."""
    rng = np.random.default_rng(seed)
    ids = [int(i) for i in rng.permutation(vocab)[:320]]
    motif = ids[0:40]
    inside = ids[40:100] + motif + ids[100:120] + motif
    distinct = [int(i) for i in rng.permutation(vocab)[:200]]
    periodic = [int(i) for i in rng.integers(0, vocab, size=10)] * 20
    outside = motif + ids[120:280] + motif
    return [inside, distinct, periodic, outside]


def _run(ng, logits: np.ndarray, seqs, n: int, window: int = WINDOW) -> np.ndarray:
    H = min(window, min(len(s) for s in seqs))
    hist = np.stack([np.asarray(s[-H:], dtype=np.int32) for s in seqs])
    out = ng.apply_ngram_guard(torch.from_numpy(logits).to(DEV), torch.from_numpy(hist).to(DEV),
                               torch.tensor([n], dtype=torch.int32, device=DEV))
    return out.cpu().numpy()


def _expect(oracle, logits, seqs, n):
    return oracle.ngram_block_rows(logits, seqs, n, WINDOW)


@pytest.mark.parametrize("n", [1, 3, 35])
def test_rows_ban_exactly_the_oracle_set(ng, oracle, n):
    seqs = _sequences(VOCAB, 0)
    logits = np.random.default_rng(5).standard_normal((4, VOCAB)).astype(np.float32)
    got = _run(ng, logits, seqs, n)
    want = _expect(oracle, logits, seqs, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    banned = [set(np.flatnonzero(got[b] == oracle.NGRAM_BLOCKED).tolist()) for b in range(4)]
    if n == 1:
        assert all(banned[b] == set(seqs[b][-WINDOW:]) for b in range(4))
    else:
        assert banned[0] and banned[2] and not banned[1] and not banned[3]
    if n == 35:
        assert banned[0] == {seqs[0][100]}  # the id after the first motif


def test_rows_do_not_mix(ng):
    seqs = _sequences(VOCAB, 1)
    logits = np.tile(np.random.default_rng(6).standard_normal(VOCAB).astype(np.float32), (4, 1))
    order = [2, 3, 0, 1]
    straight = _run(ng, logits, seqs, 3)
    swapped = _run(ng, logits, [seqs[i] for i in order], 3)
    assert np.array_equal(swapped, straight[order])
    assert not np.array_equal(straight[0], straight[2])


@pytest.mark.parametrize("n", [0, -1])
def test_n_below_one_passes_through(ng, n):
    seqs = _sequences(VOCAB, 2)
    logits = np.random.default_rng(7).standard_normal((4, VOCAB)).astype(np.float32)
    assert np.array_equal(_run(ng, logits, seqs, n), logits)


def test_a_history_shorter_than_n_bans_nothing(ng):
    seqs = _sequences(VOCAB, 3)
    logits = np.random.default_rng(8).standard_normal((4, VOCAB)).astype(np.float32)
    assert np.array_equal(_run(ng, logits, seqs, WINDOW + 1), logits)


@pytest.mark.parametrize("n", [1, 35])
def test_the_real_vocabulary_at_b8(ng, oracle, n):
    seqs = _sequences(REAL_VOCAB, 11) + _sequences(REAL_VOCAB, 13)
    logits = np.random.default_rng(12).standard_normal((8, REAL_VOCAB)).astype(np.float32)
    got = _run(ng, logits, seqs, n)
    assert np.array_equal(got.view(np.uint32), _expect(oracle, logits, seqs, n).view(np.uint32))


def test_ragged_vocabulary_long_history_and_in_place(ng, oracle):
    """V not a multiple of 4 (the unvectorised path), a history longer than the shared-memory
    stage (read from global memory), ids outside the vocabulary, and out == logits."""
    rng = np.random.default_rng(21)
    V, H, n = 1001, 9000, 3
    base = [int(i) for i in rng.integers(0, V, size=H - 6)]
    seq = base + [-5, V + 7, 4, 5, 4, 5]  # ids outside [0, V) never ban; the tail "4 5" recurs
    logits = rng.standard_normal((1, V)).astype(np.float32)
    t = torch.from_numpy(logits).to(DEV)
    hist = torch.from_numpy(np.asarray(seq, dtype=np.int32)).to(DEV)
    ng.apply_ngram_guard(t, hist.view(1, -1), torch.tensor([n], dtype=torch.int32, device=DEV), out=t)
    want = oracle.ngram_block_rows(logits, [seq], n, H)
    assert np.array_equal(t.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert t.cpu().numpy()[0, 4] == oracle.NGRAM_BLOCKED


@pytest.mark.parametrize("n", [1, 3, 35])
def test_one_row_form_matches_the_rows_form(ng, oracle, n):
    seqs = _sequences(VOCAB, 0)
    logits = np.random.default_rng(9).standard_normal((4, VOCAB)).astype(np.float32)
    rows = _run(ng, logits, seqs, n)
    blocker = ng.NgramBlocker(ngram_size=n, window=WINDOW, vocab_size=VOCAB, device=DEV)
    for b, seq in enumerate(seqs):
        got = blocker.apply(logits[b], seq)
        assert got.shape == (VOCAB,)
        assert np.array_equal(got.view(np.uint32), rows[b].view(np.uint32))
        tg = blocker.apply(torch.from_numpy(logits[b]).to(DEV), seq)
        assert np.array_equal(tg.cpu().numpy().view(np.uint32), rows[b].view(np.uint32))
