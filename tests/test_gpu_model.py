"""The Qwen2 decode and packed prefill on this package's kernels
(``PagedModelRunner``) and one GPU's serving loop (``ReplicaEngine``)
against the reference's forward with the oracle as attention, and against
transformers' own forward and greedy loop."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.qwen_reference import (random_tables, reference_decode, reference_greedy, reference_prefill_logits,
                                  small_qwen)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    torch.backends.cuda.matmul.allow_tf32 = False


def _pools(layers, num_blocks, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    shape = (layers, num_blocks, 2, 16, 64)
    return (torch.randn(shape, generator=g, device="cuda").to(dtype),
            torch.randn(shape, generator=g, device="cuda").to(dtype))


def _decode_case(dtype, seed=0):
    from pagedserve_b200.model_runner import PagedModelRunner, QwenWeights
    model = small_qwen(dtype=dtype, seed=seed)
    rng = np.random.default_rng(seed)
    lens = [1, 17, 64, 300, 1000, 2500]
    nb = sum(-(-n // 16) for n in lens) + 7
    tables = random_tables(rng, lens, nb)
    kc, vc = _pools(2, nb, dtype, seed)
    kc_ref, vc_ref = kc.clone(), vc.clone()
    positions = [n - 1 for n in lens]
    tokens = torch.tensor(rng.integers(0, model.config.vocab_size, len(lens)), device="cuda")
    want = reference_decode(model, tokens, positions, kc_ref, vc_ref, tables)
    runner = PagedModelRunner(QwenWeights.from_hf(model), kc, vc)
    width = max(len(t) for t in tables)
    table_t = torch.zeros(len(lens), width, dtype=torch.int32, device="cuda")
    for i, t in enumerate(tables):
        table_t[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    pos_t = torch.tensor(positions, dtype=torch.int64, device="cuda")
    slots = torch.tensor([t[p // 16] * 16 + p % 16 for t, p in zip(tables, positions)], device="cuda")
    got = runner.decode(tokens, pos_t, table_t, torch.tensor(lens, dtype=torch.int32, device="cuda"), slots)
    torch.cuda.synchronize()
    return got, want, (kc, vc), (kc_ref, vc_ref)


def test_decode_step_matches_reference_fp32():
    """One decode token for six fragmented requests (contexts 1 .. 2500)
    through two Qwen2.5-0.5B layers in fp32: logits and the written pools
    against transformers' modules + the oracle's attention."""
    got, want, (kc, vc), (kc_ref, vc_ref) = _decode_case(torch.float32)
    diff = (got - want).abs()
    assert diff.max().item() <= 2e-4, diff.max().item()
    # the new rows differ only by the projection GEMMs' fp32 summation order
    # (one fused q|k|v GEMM here, three in transformers); RoPE itself is exact
    torch.testing.assert_close(kc, kc_ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(vc, vc_ref, rtol=1e-5, atol=1e-5)


def test_decode_step_bf16_tracks_reference():
    """The same step in bf16: the pools' new rows match to a bf16 rounding
    and the logits stay within the spread two bf16 evaluations of the same
    model have (different GEMM shapes accumulate in different orders)."""
    got, want, (kc, vc), (kc_ref, vc_ref) = _decode_case(torch.bfloat16, seed=1)
    diff = (got.float() - want.float()).abs()
    assert diff.max().item() <= 6e-2 and diff.mean().item() <= 6e-3, (diff.max().item(), diff.mean().item())
    for a, b in ((kc, kc_ref), (vc, vc_ref)):
        torch.testing.assert_close(a.float(), b.float(), rtol=1.6e-2, atol=1.6e-2)


def test_packed_prefill_matches_transformers_fp32():
    """Three prompts (5, 130 and 700 tokens) in one packed prefill: each
    sequence's last-token logits against transformers' full forward of that
    prompt alone, and the pool rows the prefill wrote are the keys and
    values a decode then reads (a decode step after it matches too)."""
    from pagedserve_b200.model_runner import PagedModelRunner, QwenWeights
    model = small_qwen(dtype=torch.float32, seed=3)
    rng = np.random.default_rng(3)
    lens = [5, 130, 700]
    nb = sum(-(-(n + 1) // 16) for n in lens) + 3
    tables = random_tables(rng, [n + 1 for n in lens], nb)
    kc, vc = _pools(2, nb, torch.float32, 3)
    prompts = [torch.tensor(rng.integers(0, 512, n), device="cuda") for n in lens]
    runner = PagedModelRunner(QwenWeights.from_hf(model), kc, vc)
    tokens = torch.cat(prompts)
    positions = torch.cat([torch.arange(n, device="cuda") for n in lens])
    slots = torch.cat([torch.tensor([t[p // 16] * 16 + p % 16 for p in range(n)], device="cuda")
                       for t, n in zip(tables, lens)])
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")
    last = (cu[1:] - 1).long()
    got = runner.prefill(tokens, positions, slots, cu, max(lens), last)
    for i, p in enumerate(prompts):
        want = reference_prefill_logits(model, p)
        assert (got[i] - want).abs().max().item() <= 2e-4
    # one decode step on top of the prefilled pools: the next token of each prompt
    nxt = got.argmax(-1)
    width = max(len(t) for t in tables)
    table_t = torch.zeros(len(lens), width, dtype=torch.int32, device="cuda")
    for i, t in enumerate(tables):
        table_t[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    pos = torch.tensor(lens, device="cuda")
    dslots = torch.tensor([t[n // 16] * 16 + n % 16 for t, n in zip(tables, lens)], device="cuda")
    dec = runner.decode(nxt, pos, table_t, (pos + 1).to(torch.int32), dslots)
    for i, p in enumerate(prompts):
        want = reference_prefill_logits(model, torch.cat([p, nxt[i:i + 1]]))
        assert (dec[i] - want).abs().max().item() <= 2e-4


def test_engine_greedy_generation_matches_transformers_fp32():
    """The serving loop end to end (FIFO admission, packed prefill graphs,
    decode graphs with padding rows, device-side token and counter state):
    every request's tokens equal transformers' greedy continuation."""
    from pagedserve_b200.model_runner import QwenWeights
    from pagedserve_b200.serving import ReplicaEngine, ServeRequest
    model = small_qwen(dtype=torch.float32, seed=5)
    eng = ReplicaEngine(QwenWeights.from_hf(model), num_blocks=256, max_running=3, max_prefill_tokens=256,
                        max_prefill_seqs=2, max_prompt=256, max_context=512, decode_buckets=(2, 3),
                        prefill_buckets=(128, 256), record_tokens=True)
    eng.capture()
    rng = np.random.default_rng(5)
    shapes = [(3, 5), (40, 3), (100, 8), (7, 1), (60, 6), (200, 4)]
    reqs = [ServeRequest(f"r{i}", rng.integers(0, 512, n), m) for i, (n, m) in enumerate(shapes)]
    for r in reqs:
        eng.submit(r)
    done = []
    for _ in range(100):
        if not eng.has_work:
            break
        done += eng.step()
    eng.check_errors()
    eng.release()
    assert sorted(r.request_id for r in done) == sorted(r.request_id for r in reqs)
    for r in reqs:
        want = reference_greedy(model, torch.tensor(r.prompt_token_ids, device="cuda"), r.max_new_tokens)
        assert r.tokens == want, r.request_id
    assert eng.cache.used_blocks == -(-128 // 16)  # only the pad request still holds blocks


def test_engine_bf16_serving_geometry():
    """The full-size serving configuration's buckets at bf16 on a 2-layer
    model: a burst of requests runs to completion with no device error and
    every request generates exactly its budget (no EOS ids configured)."""
    from pagedserve_b200.model_runner import QwenConfig, QwenWeights
    from pagedserve_b200.serving import ReplicaEngine, ServeRequest, poisson_trace, prompt_tokens
    cfg = QwenConfig(layers=2)
    w = QwenWeights.random(cfg, "cuda", torch.bfloat16, seed=7)
    eng = ReplicaEngine(w, num_blocks=20000, max_running=64, max_prefill_tokens=4096, max_prefill_seqs=16,
                        decode_buckets=(16, 32, 64), prefill_buckets=(512, 1024, 2048, 4096))
    eng.capture()
    trace = poisson_trace(150, 1e9, seed=7, prompt_hi=2048, output_mean=20)
    reqs = [ServeRequest(f"q{i}", prompt_tokens(i, p, cfg.vocab, 7), o) for i, (_, p, o) in enumerate(trace)]
    for r in reqs:
        eng.submit(r)
    finished = []
    while eng.has_work:
        finished += eng.step()
    eng.check_errors()
    eng.release()
    assert len(finished) == len(reqs)
    assert all(r.generated == r.max_new_tokens and not r.eos for r in reqs)
    assert eng.stats["decode_tokens"] + eng.stats["first_tokens"] == sum(r.max_new_tokens for r in reqs)


def test_mixed_pass_equals_prefill_then_decode_fp32():
    """One pass over new prompts and decode rows (the serving loop's mixed
    step) gives the logits and pool rows of a packed prefill and a decode
    run apart."""
    from pagedserve_b200.model_runner import PagedModelRunner, QwenWeights
    model = small_qwen(dtype=torch.float32, seed=11)
    rng = np.random.default_rng(11)
    plens = [3, 200, 77]           # prompts
    dlens = [1, 40, 513, 1200]     # decode rows: contexts including the new token
    nb = sum(-(-n // 16) for n in plens + dlens) + 4
    tables = random_tables(rng, plens + dlens, nb)
    kc, vc = _pools(2, nb, torch.float32, 11)
    kc2, vc2 = kc.clone(), vc.clone()
    w = QwenWeights.from_hf(model)
    apart, together = PagedModelRunner(w, kc, vc), PagedModelRunner(w, kc2, vc2)
    ptab, dtab = tables[:len(plens)], tables[len(plens):]
    prompts = torch.tensor(rng.integers(0, 512, sum(plens)), device="cuda")
    ppos = torch.cat([torch.arange(n, device="cuda") for n in plens])
    pslots = torch.cat([torch.tensor([t[p // 16] * 16 + p % 16 for p in range(n)], device="cuda")
                        for t, n in zip(ptab, plens)])
    cu = torch.tensor([0] + list(np.cumsum(plens)), dtype=torch.int32, device="cuda")
    dtok = torch.tensor(rng.integers(0, 512, len(dlens)), device="cuda")
    dpos = torch.tensor([n - 1 for n in dlens], device="cuda")
    dslots = torch.tensor([t[(n - 1) // 16] * 16 + (n - 1) % 16 for t, n in zip(dtab, dlens)], device="cuda")
    width = max(len(t) for t in dtab)
    dtable = torch.zeros(len(dlens), width, dtype=torch.int32, device="cuda")
    for i, t in enumerate(dtab):
        dtable[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    dctx = torch.tensor(dlens, dtype=torch.int32, device="cuda")
    a1 = apart.prefill(prompts, ppos, pslots, cu, max(plens), (cu[1:] - 1).long())
    a2 = apart.decode(dtok, dpos, dtable, dctx, dslots)
    tp = int(sum(plens))
    last = torch.cat([(cu[1:] - 1).long(), torch.arange(tp, tp + len(dlens), device="cuda")])
    b = together.mixed(torch.cat([prompts, dtok]), torch.cat([ppos, dpos]), torch.cat([pslots, dslots]), tp, cu,
                       max(plens), dtable, dctx, last)
    torch.cuda.synchronize()
    torch.testing.assert_close(b, torch.cat([a1, a2]), rtol=1e-5, atol=1e-5)
    # the projections of a taller GEMM may sum in another fp32 order
    torch.testing.assert_close(kc2, kc, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(vc2, vc, rtol=1e-5, atol=1e-5)
