"""Greedy selection of a decode step's next tokens, on the device.

The reference ends every batched decode step with

    tokens = logits[:, -1, :].argmax(dim=-1, keepdim=True)
    for row, request in enumerate(active):
        token_id = int(tokens[row:row + 1].item())      # one sync per row
        request.add_generated_token(token_id)           # raises when none remain
        if token_id in eos_ids or request.remaining_tokens == 0:
            ...finish the request...

(pagedserve/engine/continuous_batcher.py:333-360; the same loop in
pagedserve/model/engine.py:479-491).  ``select_next_tokens`` runs the argmax,
the limit check, the countdown and the finish test for all rows in one
kernel (psb_select_tokens); ``read_selection`` brings the tokens and the
finish flags to the host with one synchronisation for the whole batch, and
raises the reference's error when a row had no tokens left.
"""

from __future__ import annotations

import threading
from typing import Iterable, Sequence

import torch

from . import ops


def eos_tensor(eos_ids: Iterable[int] | int | None, device: torch.device | str) -> torch.Tensor:
    """The reference's eos set (``generation_config.eos_token_id``: None, an
    int or a list; continuous_batcher.py:143-147) as a device int64 tensor."""
    if eos_ids is None:
        ids: list[int] = []
    elif isinstance(eos_ids, int):
        ids = [eos_ids]
    else:
        ids = sorted({int(e) for e in eos_ids})
    return torch.tensor(ids, dtype=torch.int64, device=device)


def remaining_tensor(max_new_tokens: Sequence[int], generated: Sequence[int],
                     device: torch.device | str) -> torch.Tensor:
    """Request.remaining_tokens (max_new_tokens - generated; request.py:84-85)
    per row, as the int32 device counter select_next_tokens decrements."""
    if len(max_new_tokens) != len(generated):
        raise ValueError("max_new_tokens and generated differ in length")
    return torch.tensor([int(m) - int(g) for m, g in zip(max_new_tokens, generated)], dtype=torch.int32,
                        device=device)


def select_next_tokens(logits: torch.Tensor, eos_ids: torch.Tensor, remaining: torch.Tensor,
                       error_flag: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(tokens [B, 1] int64, status [B] uint8)`` on the device, without a sync.

    ``tokens`` equals ``logits[:, -1, :].argmax(dim=-1, keepdim=True)`` (or
    ``logits.argmax(-1, keepdim=True)`` for ``[B, V]``) and can be fed to the
    next step as its input ids; ``remaining`` is decremented in place.
    """
    if not logits.is_cuda:
        raise ValueError("select_next_tokens requires CUDA tensors")
    tokens, status = ops.select_tokens(logits, eos_ids, remaining, error_flag=error_flag)
    return tokens.view(-1, 1), status


_pinned = threading.local()


def _staging(n: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Pinned host buffers for ``n`` tokens and ``n`` status bytes, kept per
    thread and grown on demand: pinning host memory costs far more than the
    copy, and read_selection's copies have completed before it returns, so
    the next call on the same thread may reuse them."""
    bufs = getattr(_pinned, "bufs", None)
    if bufs is None or bufs[0].numel() < n:
        size = max(n, 256)
        bufs = (torch.empty(size, dtype=torch.int64, pin_memory=True),
                torch.empty(size, dtype=torch.uint8, pin_memory=True))
        _pinned.bufs = bufs
    return bufs[0][:n], bufs[1][:n]


class GenerationLimitError(RuntimeError):
    """A row of the batch had no tokens left to generate.

    The reference's ``Request.add_generated_token`` raises ``RuntimeError``
    with this message (request.py:105-106) inside its per-row loop
    (continuous_batcher.py:333-360), after the rows before the failing one
    have taken their tokens.  ``row`` is the first such row; ``tokens`` and
    ``finished`` hold the whole batch's selection, so a caller can apply rows
    ``0 .. row - 1`` as the reference does.  On the device, ``remaining`` has
    already been decremented for every row that was not at its limit (rows
    at their limit keep their counter).
    """

    def __init__(self, row: int, tokens: list[int], finished: list[bool]):
        super().__init__("Request has reached its generation limit")
        self.row = row
        self.tokens = tokens
        self.finished = finished


def read_selection(tokens: torch.Tensor, status: torch.Tensor) -> tuple[list[int], list[bool]]:
    """Host copy of one step's selection: (token ids, finished flags).

    One synchronisation for the batch.  Raises ``GenerationLimitError`` (a
    ``RuntimeError`` with the reference's message, request.py:105-106) when a
    row had no tokens left; it carries the batch's tokens and flags and the
    first failing row.
    """
    if tokens.numel() != status.numel():
        raise ValueError("tokens and status differ in length")
    host_t, host_s = _staging(tokens.numel())
    host_t.copy_(tokens.reshape(-1), non_blocking=True)
    host_s.copy_(status.reshape(-1), non_blocking=True)
    torch.cuda.current_stream(tokens.device).synchronize()
    flags = host_s.tolist()
    ids = host_t.tolist()
    finished = [bool(f & ops.SELECT_DONE) for f in flags]
    for row, f in enumerate(flags):
        if f & ops.SELECT_LIMIT:
            raise GenerationLimitError(row, ids, finished)
    return ids, finished
