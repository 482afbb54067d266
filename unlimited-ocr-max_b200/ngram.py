"""The no-repeat-n-gram guard (the reference's ``ngram.py``, :1-104) on the library's kernel.

:func:`apply_ngram_guard` is the one op over all ``B`` rows (row ``b`` against row ``b`` of
``history``, the request's last ``window`` token ids); :class:`NgramBlocker` guards one row of
logits against a whole token sequence, as the reference's prefill guard does. ``ngram_size < 1``
passes the logits through unchanged, so a decode step with the guard off is the same launch fed
``n = 0``.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from .ops import ngram_block

__all__ = ["DEFAULT_NGRAM_SIZE", "BLOCKED", "NgramBlocker", "apply_ngram_guard"]

#: The reference's pairing for this model (ngram.py:30); its window is the R-SWA ring (128).
DEFAULT_NGRAM_SIZE = 35
#: What a banned logit becomes (kernels/ngram_block.mojo:47): finite, argmax- and softmax-equivalent to -inf.
BLOCKED = -3.0e38


def apply_ngram_guard(logits: torch.Tensor, history: torch.Tensor, ngram_size: torch.Tensor,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """``logits [B, V]`` (or ``[V]``) guarded against ``history [B, H]`` (or ``[H]``), ``ngram_size``
    an int32 ``[1]`` device tensor (ngram.py:34-55)."""
    return ngram_block(logits, history, ngram_size, out=out)


class NgramBlocker:
    """One row of logits against a whole sequence (ngram.py:57-104): the sequence's last
    ``window`` ids are the history; a sequence shorter than ``ngram_size`` bans nothing."""

    def __init__(self, *, ngram_size: int, window: int, vocab_size: int, device: str | torch.device = "cuda"):
        if ngram_size < 1 or window < 1:
            raise ValueError("ngram_size and window must be >= 1")
        self.ngram_size, self.window, self.vocab_size = int(ngram_size), int(window), int(vocab_size)
        self.device = torch.device(device)
        self._ngram = torch.tensor([self.ngram_size], dtype=torch.int32, device=self.device)

    def apply(self, logits, sequence: Sequence[int]):
        """``logits`` (a CUDA tensor or a numpy array of ``vocab_size`` fp32) with every banned id set
        to :data:`BLOCKED`; returned as the type it came in."""
        ids = np.asarray(sequence, dtype=np.int32).reshape(-1)
        as_numpy = isinstance(logits, np.ndarray)
        flat = torch.from_numpy(np.ascontiguousarray(logits, dtype=np.float32).reshape(-1)).to(self.device) \
            if as_numpy else logits.reshape(-1)
        if flat.shape[0] != self.vocab_size:
            raise ValueError(f"logits has {flat.shape[0]} entries, expected {self.vocab_size}")
        if ids.shape[0] < self.ngram_size:
            return logits
        history = torch.from_numpy(np.ascontiguousarray(ids[-self.window:])).to(self.device)
        got = ngram_block(flat.to(torch.float32), history, self._ngram)
        return got.cpu().numpy() if as_numpy else got
