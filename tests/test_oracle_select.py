"""The selection oracle on the CPU: pinned to the reference's own argmax
expression and Request bookkeeping (golden vectors from
tests/golden/make_golden_select.py), and to torch.argmax on edge cases."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import select_tokens as sel

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "select_outputs.npz"))


@pytest.mark.parametrize("name", ["bf16", "f16", "f32", "bf16_ties"])
def test_oracle_matches_reference_selection(name):
    tokens, status, rem, limit = sel.select_tokens(GOLD[f"{name}/logits"][:, -1], GOLD["eos_ids"],
                                                   GOLD[f"{name}/remaining"])
    assert np.array_equal(tokens, GOLD[f"{name}/tokens"])
    assert np.array_equal(status, GOLD[f"{name}/status"])
    assert np.array_equal(rem, GOLD[f"{name}/remaining_after"])
    assert limit == bool(np.any(GOLD[f"{name}/status"] & sel.LIMIT))


def test_golden_covers_every_outcome():
    status = np.concatenate([GOLD[f"{n}/status"] for n in ("bf16", "f16", "f32", "bf16_ties")])
    assert {0, sel.DONE, sel.DONE | sel.EOS, sel.DONE | sel.LIMIT} <= set(int(s) for s in status)


def _edge_rows(v: int, rng) -> np.ndarray:
    rows = rng.standard_normal((10, v)).astype(np.float32)
    rows[0] = -np.inf
    rows[1, [v - 1, 3 % v]] = np.nan
    rows[2] = 0.0
    rows[2, : v // 2] = -0.0
    rows[3, [1 % v, v - 1]] = np.inf
    rows[4] = 7.0
    rows[5, v - 1] = 50.0
    rows[6, :] = -np.inf
    rows[6, v - 1] = -3e38
    rows[7, 0] = np.nan
    rows[8] = np.round(rows[8])  # many ties
    rows[9, [v // 2, (v // 2 + 1) % v]] = 100.0
    return rows


@pytest.mark.parametrize("v", [1, 2, 7, 64, 1000, 4099])
def test_argmax_first_equals_torch(v):
    rows = _edge_rows(v, np.random.default_rng(v))
    want = torch.from_numpy(rows).argmax(dim=-1).numpy()
    assert np.array_equal(sel.argmax_first(rows), want)
    for dt in (torch.bfloat16, torch.float16):
        r = torch.from_numpy(rows).to(dt)
        assert np.array_equal(sel.argmax_first(r.float().numpy()), r.argmax(dim=-1).numpy())


def test_countdown_and_stop():
    rows = np.zeros((4, 8), dtype=np.float32)
    rows[:, 2] = 1.0
    rows[1, 2], rows[1, 5] = 0.0, 1.0
    tokens, status, rem, limit = sel.select_tokens(rows, [2], np.array([3, 3, 1, 0], dtype=np.int32))
    assert tokens.tolist() == [2, 5, 2, 2]
    assert status.tolist() == [sel.DONE | sel.EOS, 0, sel.DONE | sel.EOS, sel.DONE | sel.LIMIT]
    assert rem.tolist() == [2, 2, 0, 0]
    assert limit
