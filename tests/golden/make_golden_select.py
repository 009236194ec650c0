"""Golden vectors for the device-side greedy selection, from the reference's code.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden_select.py --reference <PagedServe checkout>

For seeded [B, S, V] logits (with planted ties, NaNs, infinities, signed
zeros and all--inf rows) this evaluates the reference's own expression
``logits[:, -1, :].argmax(dim=-1, keepdim=True)``
(pagedserve/engine/continuous_batcher.py:333-335) with torch on the CPU, and
runs each row through the reference's ``Request`` class
(pagedserve/engine/request.py): ``add_generated_token`` (which raises when no
tokens remain) and the finish test ``token_id in eos_ids or
request.remaining_tokens == 0`` (continuous_batcher.py:337-360).  Inputs and
outputs go to ``tests/golden/select_outputs.npz``; nothing on the GPU box
reads the reference.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, dtype, batch, positions, vocab)
CASES = [("bf16", "bfloat16", 12, 2, 1000), ("f16", "float16", 10, 1, 777), ("f32", "float32", 9, 3, 64),
         ("bf16_ties", "bfloat16", 16, 1, 40)]
EOS = [2, 7, 151643]


def plant(logits, rng):
    """Edge cases in the last position of some rows (bit patterns the kernels
    must rank exactly as torch does)."""
    b, _, v = logits.shape
    last = logits[:, -1]
    last[0, :] = -np.inf                                  # all -inf: index 0
    last[1, v // 3] = np.nan                              # one NaN
    last[1, v // 2] = np.inf
    last[2, 5] = np.inf                                   # first +inf of two
    last[2, v - 1] = np.inf
    last[3, :] = 0.0                                      # signed zeros, equal
    last[3, : v // 2] = -0.0
    last[4, [v - 3, 3]] = np.nan                          # first NaN by index
    last[5, :] = -1.0                                     # all equal: index 0
    last[6, v - 1] = 1e4                                  # max at the last index
    last[7, 2] = 1e4                                      # an EOS id wins
    if b > 8:
        last[8, :] = -np.inf
        last[8, v - 2] = -1e30                            # one finite value
    return logits


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of a PagedServe checkout (the directory holding the pagedserve package)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)

    import torch
    from pagedserve.engine.request import Request, RequestStatus

    dtypes = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
    arrays: dict[str, np.ndarray] = {}
    for i, (name, dtype, b, s, v) in enumerate(CASES):
        rng = np.random.default_rng(200 + i)
        if name.endswith("ties"):
            # few distinct values: many rows tie on their maximum
            logits = rng.integers(-3, 3, size=(b, s, v)).astype(np.float32)
        else:
            logits = (3.0 * rng.standard_normal((b, s, v))).astype(np.float32)
        logits = plant(logits, rng)
        lt = torch.from_numpy(logits).to(dtypes[dtype])
        tokens = lt[:, -1, :].argmax(dim=-1, keepdim=True)          # the reference's expression
        max_new = rng.integers(1, 6, size=b)
        generated = np.minimum(rng.integers(0, 6, size=b), max_new)
        status = np.zeros(b, dtype=np.uint8)
        remaining_after = np.zeros(b, dtype=np.int32)
        for row in range(b):
            req = Request(request_id=f"r{row}", prompt_token_ids=[1, 2, 3], max_new_tokens=int(max_new[row]),
                          generated_token_ids=[9] * int(generated[row]))
            req.transition(RequestStatus.RUNNING)
            remaining_before = req.remaining_tokens
            token_id = int(tokens[row:row + 1].item())
            try:
                req.add_generated_token(token_id)
            except RuntimeError:
                status[row] = 1 | 4
                remaining_after[row] = remaining_before
                continue
            eos = token_id in EOS
            status[row] = (1 if (eos or req.remaining_tokens == 0) else 0) | (2 if eos else 0)
            remaining_after[row] = req.remaining_tokens
        arrays[f"{name}/logits"] = lt.float().numpy()
        arrays[f"{name}/remaining"] = (max_new - generated).astype(np.int32)
        arrays[f"{name}/tokens"] = tokens[:, 0].numpy().astype(np.int64)
        arrays[f"{name}/status"] = status
        arrays[f"{name}/remaining_after"] = remaining_after
    arrays["eos_ids"] = np.array(EOS, dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "select_outputs.npz"), **arrays)
    print(f"wrote {len(arrays)} arrays")


if __name__ == "__main__":
    main()
