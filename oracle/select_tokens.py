"""CPU oracle for the device-side greedy selection.  TEST INFRASTRUCTURE ONLY.

Restates in numpy what PagedServe does with a decode step's logits:

* ``argmax_first``   <- ``logits[:, -1, :].argmax(dim=-1, keepdim=True)``
                        (pagedserve/engine/continuous_batcher.py:333-335,
                        pagedserve/model/engine.py:479): torch's argmax - the
                        first index of the maximum, any NaN larger than every
                        number (the first NaN wins), -0.0 equal to +0.0.
* ``select_tokens``  <- the per-row loop after it
                        (pagedserve/engine/continuous_batcher.py:337-360):
                        ``request.add_generated_token(token_id)`` raises when
                        ``remaining_tokens <= 0`` (pagedserve/engine/request.py:99-106),
                        else the request finishes when
                        ``token_id in eos_ids or request.remaining_tokens == 0``
                        with ``remaining_tokens = max_new_tokens - generated``
                        (request.py:84-85).

Imported only by ``tests/``.  Parity is pinned by
``tests/golden/make_golden_select.py``, which runs torch's argmax on the
reference's expression and the reference's own ``Request`` class on seeded
rows and stores the results in ``tests/golden/select_outputs.npz``.
"""

from __future__ import annotations

import numpy as np

DONE, EOS, LIMIT = 1, 2, 4


def argmax_first(rows: np.ndarray) -> np.ndarray:
    """Index of the first maximum of each row; NaN beats every number.
    rows: [B, V] float array (any float dtype) -> [B] int64."""
    rows = np.asarray(rows, dtype=np.float64)
    out = np.empty(rows.shape[0], dtype=np.int64)
    for b, r in enumerate(rows):
        nan = np.flatnonzero(np.isnan(r))
        if nan.size:
            out[b] = nan[0]
        else:
            # np.argmax returns the first maximum; -0.0 == +0.0 compares equal
            out[b] = int(np.argmax(r))
    return out


def select_tokens(rows: np.ndarray, eos_ids, remaining: np.ndarray):
    """(tokens [B] int64, status [B] uint8, remaining after [B] int32,
    limit error raised) for one step, as the reference's loop leaves them."""
    tokens = argmax_first(rows)
    rem = np.asarray(remaining, dtype=np.int32).copy()
    status = np.zeros(len(tokens), dtype=np.uint8)
    eos = {int(e) for e in eos_ids}
    limit = False
    for b, tok in enumerate(tokens):
        if rem[b] <= 0:              # add_generated_token raises
            limit = True
            status[b] = DONE | LIMIT
            continue
        rem[b] -= 1
        is_eos = int(tok) in eos
        status[b] = (DONE if (is_eos or rem[b] == 0) else 0) | (EOS if is_eos else 0)
    return tokens, status, rem, limit
