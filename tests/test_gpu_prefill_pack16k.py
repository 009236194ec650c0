"""Parity at the size the prefill benchmark times: the four 16K-token packs
of prompts lognormal(median 256, sigma 1.0) clipped to [32, 2048] (seeds
2000-2003), every sequence checked.

Per pack: the fused RoPE + paged KV write (bit-exact against the oracle's
restatement of apply_rotary_pos_emb + write_token), then the packed prefill
(varlen_prefill), the same prompts read back from the pool (paged_prefill)
and each prompt's second half prefilled over its first half (chunked,
paged_prefill with a prefix) against the float64 oracle of the reference's
causal attention (paged_attention.py:94-145).  The pools hold NaN outside
every written slot, so a read outside a context shows up."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import paged_attention as ora
from tests.helpers import err_stats

pytestmark = pytest.mark.gpu

HQ, HKV, D, BS = 14, 2, 64, 16


def pack_lengths(seed: int, tokens: int = 16384) -> list[int]:
    """The benchmark's packs: lognormal(256, 1.0) prompts in [32, 2048], packed up to 16384 tokens."""
    rng = np.random.default_rng(seed)
    lens = []
    while True:
        n = int(np.clip(round(rng.lognormal(math.log(256), 1.0)), 32, 2048))
        if sum(lens) + n > tokens:
            return lens
        lens.append(n)


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


@pytest.mark.parametrize("seed", [2000, 2001, 2002, 2003])
def test_full_pack_rope_write_prefill_paged_chunked(seed):
    from pagedserve_b200 import ops
    lens = pack_lengths(seed)
    t = sum(lens)
    assert t > 14000 and max(lens) <= 2048
    rng = np.random.default_rng(seed)
    q = ora.bf16_round(rng.standard_normal((t, HQ, D), dtype=np.float32))
    k = ora.bf16_round(rng.standard_normal((t, HKV, D), dtype=np.float32))
    v = ora.bf16_round(rng.standard_normal((t, HKV, D), dtype=np.float32))
    pos = np.concatenate([np.arange(n) for n in lens]).astype(np.float32)
    inv = 1.0 / (1e6 ** (np.arange(0, D, 2, dtype=np.float32) / D))
    ang = np.concatenate([np.outer(pos, inv)] * 2, axis=1)
    cos, sin = ora.bf16_round(np.cos(ang)), ora.bf16_round(np.sin(ang))
    need = [-(-n // BS) for n in lens]
    nb = int(sum(need) * 1.25)
    perm = rng.permutation(nb)
    tables, at = [], 0
    for c in need:
        tables.append(perm[at:at + c].tolist())
        at += c
    slots = ora.slot_mapping(tables, [list(range(n)) for n in lens], BS)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)

    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)
    kc = torch.full((1, nb, HKV, BS, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    vc = torch.full_like(kc, float("nan"))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    q_rot, k_rot = ops.rope_reshape_and_cache(bf(q), bf(k), bf(v), bf(cos), bf(sin), kc, vc,
                                              torch.from_numpy(slots).cuda(), 0, error_flag=err)
    cu_t = torch.from_numpy(cu).cuda()
    table_t = torch.from_numpy(ora.padded_block_table(tables)).cuda()
    ctx_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = ops.varlen_prefill(q_rot, k_rot, bf(v), cu_t, max(lens), error_flag=err)
    paged = ops.paged_prefill(q_rot, kc, vc, table_t, ctx_t, cu_t, max(lens), 0, error_flag=err)
    chunks = [n - n // 2 for n in lens]
    rows = np.concatenate([np.arange(a + n // 2, a + n) for a, n in zip(cu[:-1], lens)])
    rows_t = torch.from_numpy(rows).cuda()
    ccu = torch.from_numpy(np.concatenate([[0], np.cumsum(chunks)]).astype(np.int32)).cuda()
    chunked = ops.paged_prefill(q_rot.index_select(0, rows_t), kc, vc, table_t, ctx_t, ccu, max(chunks), 0,
                                error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0

    # RoPE + write: bit-exact, every token, every pool slot
    kc_want = np.full((1, nb, HKV, BS, D), np.nan, dtype=np.float32)
    vc_want = kc_want.copy()
    q_want, k_want = ora.rope_reshape_and_cache(q, k, v, cos, sin, kc_want, vc_want, slots, 0, "bfloat16")
    assert np.array_equal(q_rot.float().cpu().numpy(), q_want)
    assert np.array_equal(k_rot.float().cpu().numpy(), k_want)
    np.testing.assert_array_equal(kc.float().cpu().numpy(), kc_want)
    np.testing.assert_array_equal(vc.float().cpu().numpy(), vc_want)

    # attention: every sequence of the pack against the float64 oracle
    exact = ora.varlen_causal_attention_blocked(q_want, k_want, v, cu)
    for name, got, want in (("varlen", out, exact), ("paged", paged, exact), ("chunked", chunked, exact[rows])):
        assert not torch.isnan(got).any(), name
        mx, mean = err_stats(got, want)
        assert mx <= 2e-2 and mean <= 2e-3, (name, mx, mean)
        # and sequence by sequence, so one bad short sequence cannot hide in the pack's mean
        g = got.float().cpu().numpy()
        starts = cu[:-1] if name != "chunked" else np.concatenate([[0], np.cumsum(chunks)])[:-1]
        sizes = lens if name != "chunked" else chunks
        for i, (a, n) in enumerate(zip(starts, sizes)):
            d = np.abs(g[a:a + n] - want[a:a + n])
            assert d.max() <= 2e-2 and d.mean() <= 2e-3, (name, i, d.max(), d.mean())
