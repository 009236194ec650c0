#!/usr/bin/env python
"""Serving-scale paged decode + reshape_and_cache on B200 (sm_100a).

Workload (one "step" = one layer call of the decode hot path over one batch):
256 sequences, context lengths lognormal(median 1024, sigma 0.8) clipped to
[16, 8192]; Qwen2.5-0.5B attention geometry (14 q heads, 2 kv heads, head_dim
64), block_size 16, bf16; physical blocks shuffled across a pool of 1.25x
the need; the step writes one new token per sequence into the pool and runs
split-K paged decode attention over it - one fused launch that stores each
row's token at its last position through the block table (the slot the
reshape_and_cache slot mapping names) - plus the split-K combine.
Synthetic seeded data (no dataset or weights are involved).  The pool holds
the model's 24 layers and consecutive steps are consecutive layers, so every
step streams ~180 MB of KV that is not resident in the 126 MB L2.  Steps run
as the decode iteration runs them: one CUDA graph holds the 24 layer calls.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Under torchrun with N ranks, N x 256 requests are drawn and placed on the
GPUs in arrival order by ``SequenceDispatcher`` (the rank with the most free
KV blocks takes the next request); each rank serves its shard from its own
pool, with no collective on the data path (weak scaling).  The step time is
the max over ranks and the bytes are summed over ranks.  ``--impl reference``
times the reference algorithm's CPU restatement (the oracle) on the host
cores instead.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BATCH, MEDIAN, SIGMA, LO, HI = 256, 1024, 0.8, 16, 8192
HQ, HKV, D, BS, SLACK = 14, 2, 64, 16, 1.25
LAYERS = 24  # Qwen2.5-0.5B decoder layers: one decode iteration is 24 layer calls
METRIC = "paged-decode attn HBM GB/s (% of ~8 TB/s); decode tok/s at 1/2/4/8 B200"
WORKLOAD_SEED = 1000  # context lengths of the decode batch, for the B200 arm and both CPU arms
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
# DRAM bytes of one fused decode step (decode with the new-token store + combine)
# on the rank-0 workload, measured with ncu
STEP_TRAFFIC_BYTES = 197_900_000


def context_lengths(seed: int, n: int = BATCH) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.clip(np.round(rng.lognormal(math.log(MEDIAN), SIGMA, n)), LO, HI).astype(np.int64)


def rank_lengths(world: int, rank: int) -> np.ndarray:
    """This rank's contexts: world x 256 requests drawn once, placed on the
    ranks in arrival order by ``SequenceDispatcher`` (most free KV blocks
    first).  At one GPU this is the plain 256-sequence batch."""
    from pagedserve_b200.sharding import shard_sequences
    lens = context_lengths(WORKLOAD_SEED, BATCH * world)
    if world == 1:
        return lens
    blocks = int(math.ceil(SLACK * np.sum(-(-lens // BS)) / world))
    return lens[shard_sequences(lens, world, blocks, BS)[rank]]


def decode_bytes(lens: np.ndarray) -> int:
    """Algorithmic HBM bytes of one decode launch: K+V of every context token
    (Hkv*D*2 B each for K and for V = 512 B/token), Q in + O out (Hq*D*2 B
    each = 3584 B/sequence), the used block-table entries and the lengths."""
    blocks = int(np.sum(-(-lens // BS)))
    return int(512 * lens.sum() + 3584 * len(lens) + 4 * blocks + 4 * len(lens))


def reshape_bytes(n_tokens: int) -> int:
    """read K+V (2*Hkv*D*2 B) + write K+V + 8 B slot = 1032 B per token."""
    return 1032 * n_tokens


def load_peaks() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_tensor_peak() -> tuple[float, str]:
    """bf16 dense TFLOP/s of a burst (the prefill kernel is timed on its own)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


PREFILL_TOKENS, PREFILL_MEDIAN, PREFILL_SIGMA, PREFILL_LO, PREFILL_HI, PREFILL_PACKS = 16384, 256, 1.0, 32, 2048, 4


def prefill_lengths(seed: int) -> list[int]:
    """Prompts lognormal(median 256, sigma 1.0) clipped to [32, 2048], packed up to 16384 tokens."""
    rng = np.random.default_rng(seed)
    lens = []
    while True:
        n = int(np.clip(round(rng.lognormal(math.log(PREFILL_MEDIAN), PREFILL_SIGMA)), PREFILL_LO, PREFILL_HI))
        if sum(lens) + n > PREFILL_TOKENS:
            return lens
        lens.append(n)


def prefill_flops(lens) -> float:
    """Causal attention FLOPs: 2 matmuls x 2 flop x Hq x D x L (L + 1) / 2 per sequence."""
    return float(sum(4 * HQ * D * n * (n + 1) / 2 for n in lens))


def chunk_flops(lens, chunks) -> float:
    """FLOPs of prefilling the last ``c`` rows of an ``n``-token context: row
    ``i`` of the chunk sees ``n - c + i + 1`` keys."""
    return float(sum(4 * HQ * D * (c * (n - c) + c * (c + 1) / 2) for n, c in zip(lens, chunks)))


def rope_cache_bytes(n_tokens: int) -> int:
    """Algorithmic bytes of rope_reshape_and_cache per token: read q, k, v, the
    cos and sin rows and the slot; write the rotated q and k and the pool's
    k and v rows (2568 + 2560 B for 14q/2kv heads, D 64, bf16)."""
    row = D * 2
    reads = (HQ + 2 * HKV) * row + 2 * row + 8
    writes = (HQ + HKV) * row + 2 * HKV * row
    return n_tokens * (reads + writes)


def run_prefill(args, device, seed: int) -> dict:
    """Packed causal prefill of one engine iteration: the fused RoPE + paged KV
    write of every prompt token (rope_reshape_and_cache), then varlen_prefill
    over the rotated q and k, on PREFILL_PACKS different packs in turn so
    consecutive steps do not run from L2."""
    from pagedserve_b200 import ops
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    packs = []
    for i in range(PREFILL_PACKS):
        lens = prefill_lengths(seed + i)
        t = sum(lens)
        need = sum(-(-n // BS) for n in lens)
        nb = int(math.ceil(SLACK * need))
        perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed + i))[:need]
        slots, at = [], 0
        table = torch.zeros(len(lens), max(-(-n // BS) for n in lens), dtype=torch.int32)
        for i, n in enumerate(lens):
            k = -(-n // BS)
            blocks = perm[at:at + k]
            table[i, :k] = blocks.to(torch.int32)
            at += k
            pos = torch.arange(n)
            slots.append(blocks[pos // BS] * BS + pos % BS)
        # chunked prefill: each prompt's second half attends over its first half
        chunks = [n - n // 2 for n in lens]
        rows = torch.cat([torch.arange(a + n // 2, a + n) for a, n in zip(np.cumsum([0] + lens[:-1]), lens)])
        # the engine's position embeddings: Qwen2 rope (theta 1e6) angles in
        # fp32, cos/sin rounded to the model dtype, one row per token
        pos = torch.cat([torch.arange(n) for n in lens]).to(device=device, dtype=torch.float32)
        inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))
        ang = torch.outer(pos, inv).repeat(1, 2)
        packs.append(dict(
            table=table.to(device), ctx=torch.tensor(lens, dtype=torch.int32, device=device), chunks=chunks,
            chunk_rows=rows.to(device), chunk_cu=torch.tensor([0] + list(np.cumsum(chunks)), dtype=torch.int32,
                                                              device=device),
            cos=ang.cos().to(torch.bfloat16), sin=ang.sin().to(torch.bfloat16),
            q_rot=torch.empty(t, HQ, D, device=device, dtype=torch.bfloat16),
            k_rot=torch.empty(t, HKV, D, device=device, dtype=torch.bfloat16),
            lens=lens, q=torch.randn(t, HQ, D, device=device, dtype=torch.bfloat16, generator=gen),
            k=torch.randn(t, HKV, D, device=device, dtype=torch.bfloat16, generator=gen),
            v=torch.randn(t, HKV, D, device=device, dtype=torch.bfloat16, generator=gen),
            cu=torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=device),
            slots=torch.cat(slots).to(device=device, dtype=torch.int64),
            kc=torch.empty(1, nb, HKV, BS, D, device=device, dtype=torch.bfloat16),
            vc=torch.empty(1, nb, HKV, BS, D, device=device, dtype=torch.bfloat16),
            out=torch.empty(t, HQ, D, device=device, dtype=torch.bfloat16)))

    def step(pk, attn=True, write=True):
        if write:
            ops.rope_reshape_and_cache(pk["q"], pk["k"], pk["v"], pk["cos"], pk["sin"], pk["kc"], pk["vc"],
                                       pk["slots"], 0, query_out=pk["q_rot"], key_out=pk["k_rot"])
        if attn:
            ops.varlen_prefill(pk["q_rot"], pk["k_rot"], pk["v"], pk["cu"], max(pk["lens"]), out=pk["out"])

    def paged(pk):  # the same prompts with K/V read from the pool through the tables
        ops.paged_prefill(pk["q_rot"], pk["kc"], pk["vc"], pk["table"], pk["ctx"], pk["cu"], max(pk["lens"]), 0,
                          out=pk["out"])

    def chunked(pk):  # each prompt's second half over its first half, from the pool
        ops.paged_prefill(pk["q_chunk"], pk["kc"], pk["vc"], pk["table"], pk["ctx"], pk["chunk_cu"],
                          max(pk["chunks"]), 0, out=pk["out_chunk"])

    stream = torch.cuda.Stream(device)
    graphs, attn_graphs, rope_graphs, paged_graphs, chunk_graphs = [], [], [], [], []
    with torch.cuda.stream(stream):
        for pk in packs:
            step(pk)
            pk["q_chunk"] = pk["q_rot"].index_select(0, pk["chunk_rows"])
            pk["out_chunk"] = torch.empty_like(pk["q_chunk"])
        torch.cuda.synchronize()
        for pk in packs:
            for lst, fn in ((graphs, lambda: step(pk)), (attn_graphs, lambda: step(pk, write=False)),
                            (rope_graphs, lambda: step(pk, attn=False)), (paged_graphs, lambda: paged(pk)),
                            (chunk_graphs, lambda: chunked(pk))):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    fn()
                lst.append(g)
    torch.cuda.synchronize()

    def timed(gs):
        for i in range(args.warmup):
            gs[i % PREFILL_PACKS].replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(args.steps):
            gs[i % PREFILL_PACKS].replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / args.steps

    step_ms, attn_ms, rope_ms = timed(graphs), timed(attn_graphs), timed(rope_graphs)
    paged_ms, chunk_ms = timed(paged_graphs), timed(chunk_graphs)
    for g in graphs + attn_graphs + rope_graphs + paged_graphs + chunk_graphs:
        g.reset()
    flops = statistics.mean(prefill_flops(pk["lens"]) for pk in packs)
    tokens = statistics.mean(sum(pk["lens"]) for pk in packs)
    peak, kind = load_tensor_peak()
    tflops = flops / (attn_ms * 1e-3) / 1e12
    rope_bytes = statistics.mean(rope_cache_bytes(sum(pk["lens"])) for pk in packs)
    hbm_peak, hbm_kind = load_peaks()
    rope_gbs = rope_bytes / (rope_ms * 1e-3) / 1e9
    cflops = statistics.mean(chunk_flops(pk["lens"], pk["chunks"]) for pk in packs)
    paged_tf, chunk_tf = flops / (paged_ms * 1e-3) / 1e12, cflops / (chunk_ms * 1e-3) / 1e12
    return {
        "workload": "packed causal prefill + fused RoPE and paged KV write: prompts lognormal(median 256, sigma "
                    "1.0) clipped [32, 2048], packed to <= 16384 tokens, 14q/2kv heads, d64, block 16, bf16, "
                    f"rope theta 1e6; {PREFILL_PACKS} packs in turn",
        "seqs_per_pack": [len(pk["lens"]) for pk in packs], "tokens_per_pack": tokens,
        "ms_per_step": round(step_ms, 5), "attn_layer_tokens_per_s": round(tokens / (step_ms * 1e-3), 1),
        "attention": {"kernel": "prefill_tc_kernel (tcgen05/TMEM, TMA)", "ms": round(attn_ms, 5),
                      "gflop": round(flops / 1e9, 3), "tflops": round(tflops, 1), "peak_tflops": peak,
                      "peak_kind": kind, "frac": round(tflops / peak, 4), "bound": "tensor"},
        "paged_attention": {"kernel": "prefill_tc_kernel<paged> (K/V from the pool through the block tables)",
                            "ms": round(paged_ms, 5), "tflops": round(paged_tf, 1), "frac": round(paged_tf / peak, 4)},
        "chunked_attention": {"workload": "each prompt's second half prefilled over its first half (prefix read "
                                          "from the pool)", "ms": round(chunk_ms, 5),
                              "gflop": round(cflops / 1e9, 3), "tflops": round(chunk_tf, 1),
                              "frac": round(chunk_tf / peak, 4)},
        "rope_cache": {"kernel": "rope_cache_kernel (RoPE of q and k + slot-mapped K/V write)",
                       "ms": round(rope_ms, 5), "mbytes": round(rope_bytes / 1e6, 2),
                       "gbs": round(rope_gbs, 1), "peak_gbs": hbm_peak, "peak_kind": hbm_kind,
                       "frac": round(rope_gbs / hbm_peak, 4), "bound": "hbm"},
        "gpu_launches_per_step": 2,
    }


VOCAB = 151936        # Qwen2.5-0.5B vocabulary (tied embeddings)
SELECT_BATCHES = (128, 256)  # greedy-sampling serving batch; this bench's decode batch
SELECT_LAUNCHES = 8   # launches per captured graph, rotating over buffers larger than L2 together


def run_select(args, device, seed: int) -> dict:
    """Greedy selection of a decode step (select_tokens: argmax over the
    vocabulary + EOS / remaining-token stop test) for the serving batches,
    bf16 logits.  Each timed graph rotates over enough logits buffers that
    together exceed the L2, so every launch streams its rows from HBM."""
    from pagedserve_b200 import ops
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    eos = torch.tensor([151643, 151645], dtype=torch.int64, device=device)
    hbm_peak, hbm_kind = load_peaks()
    out = {"kernel": "select_stream_kernel (persistent thread-block clusters, bulk async copies into per-warp "
                     "shared-memory slots, DSMEM merge)",
           "workload": f"bf16 logits [B, {VOCAB}], EOS ids {{151643, 151645}}, remaining counters; buffers rotated "
                       "so each graph's launches read > 126 MB", "batches": {}}
    for batch in SELECT_BATCHES:
        row_bytes = VOCAB * 2
        nbuf = max(2, -(-200_000_000 // (batch * row_bytes)))
        bufs = [torch.randn(batch, VOCAB, device=device, generator=gen).to(torch.bfloat16) for _ in range(nbuf)]
        rem = torch.full((batch,), 1 << 30, dtype=torch.int32, device=device)
        tokens = torch.empty(batch, dtype=torch.int64, device=device)
        status = torch.empty(batch, dtype=torch.uint8, device=device)
        nbytes = batch * row_bytes + batch * (8 + 1 + 2 * 4) + eos.numel() * 8
        res = {"mbytes_per_launch": round(nbytes / 1e6, 3)}
        stream = torch.cuda.Stream(device)
        for ctas in (0, 1, 2, 4, 6, 8):
            with torch.cuda.stream(stream):
                ops.select_tokens(bufs[0], eos, rem, tokens=tokens, status=status, ctas_per_row=ctas)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for i in range(SELECT_LAUNCHES):
                        ops.select_tokens(bufs[i % nbuf], eos, rem, tokens=tokens, status=status,
                                          ctas_per_row=ctas)
            for _ in range(args.warmup):
                g.replay()
            torch.cuda.synchronize()
            reps = max(1, args.steps // SELECT_LAUNCHES)
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(reps):
                g.replay()
            e.record()
            torch.cuda.synchronize()
            g.reset()
            ms = a.elapsed_time(e) / (reps * SELECT_LAUNCHES)
            gbs = nbytes / (ms * 1e-3) / 1e9
            res["auto" if ctas == 0 else f"ctas{ctas}"] = {"us": round(ms * 1e3, 3), "gbs": round(gbs, 1),
                                                           "frac": round(gbs / hbm_peak, 4)}
        # the reference's own expression, logits.argmax(dim=-1), on the same buffers
        with torch.cuda.stream(stream):
            torch.argmax(bufs[0], dim=-1, out=tokens)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(SELECT_LAUNCHES):
                    torch.argmax(bufs[i % nbuf], dim=-1, out=tokens)
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        reps = max(1, args.steps // SELECT_LAUNCHES)
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        e.record()
        torch.cuda.synchronize()
        g.reset()
        res["torch_argmax_us"] = round(a.elapsed_time(e) / (reps * SELECT_LAUNCHES) * 1e3, 3)
        # correctness of the timed configuration against torch on the last buffer
        rem.fill_(1 << 30)
        ops.select_tokens(bufs[-1], eos, rem, tokens=tokens, status=status)
        res["matches_torch_argmax"] = bool(torch.equal(tokens, bufs[-1].argmax(dim=-1)))
        out["batches"][str(batch)] = res
        del bufs
    out.update({"peak_gbs": hbm_peak, "peak_kind": hbm_kind, "bound": "hbm"})
    return out


# ---------------------------------------------------------------------------
# model-level decode: a whole Qwen2.5-0.5B decode iteration (config 3)
# ---------------------------------------------------------------------------
MODEL_BATCH, MODEL_MEDIAN, MODEL_SIGMA = 128, 512, 0.8
EOS_IDS = (151643, 151645)  # Qwen2.5's end-of-text ids


def model_context_lengths(seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.clip(np.round(rng.lognormal(math.log(MODEL_MEDIAN), MODEL_SIGMA, MODEL_BATCH)), LO, HI).astype(np.int64)


def run_model_decode(args, device, seed: int) -> dict:
    """One decode iteration of random-init Qwen2.5-0.5B (24 layers, bf16) for
    128 sequences with lognormal(median 512, sigma 0.8) contexts over a
    shuffled paged pool: pack_step, embedding, 24 x (RMSNorm, fused QKV GEMM,
    RoPE + KV write, split-K paged decode, o_proj, residual + RMSNorm, fused
    gate/up GEMM, SiLU * up, down GEMM), final norm, tied lm_head, greedy
    selection - one captured graph, the serving loop's decode step."""
    from pagedserve_b200 import ops
    from pagedserve_b200.model_runner import QwenConfig, QwenWeights
    from pagedserve_b200.serving import ReplicaEngine, _BIG_REMAINING
    cfg = QwenConfig()
    w = QwenWeights.random(cfg, device, torch.bfloat16, seed=seed)
    lens = model_context_lengths(seed)
    rng = np.random.default_rng(seed + 1)
    need = int(np.sum(-(-(lens + 1) // BS))) + 8
    nb = int(math.ceil(SLACK * need))
    eng = ReplicaEngine(w, nb, max_running=MODEL_BATCH, max_prefill_tokens=512, max_prompt=512,
                        decode_buckets=(MODEL_BATCH,), prefill_buckets=(512,), free_order=rng.permutation(nb))
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    eng.cache.kv_cache.k_cache.normal_(generator=gen)
    eng.cache.kv_cache.v_cache.normal_(generator=gen)
    ids = [f"m{i}" for i in range(MODEL_BATCH)]
    for rid, n in zip(ids, lens):
        eng.cache.allocate(rid, int(n) + 1)
    eng._upload_tables(ids)
    rows = np.array([eng._store_row(r) for r in ids], dtype=np.int32)
    rows_t = torch.from_numpy(rows.astype(np.int64)).to(device)
    eng.remaining[rows_t] = _BIG_REMAINING
    eng.last_token[rows_t] = torch.randint(0, cfg.vocab, (MODEL_BATCH,), generator=gen, device=device)
    g = eng._decode[MODEL_BATCH]
    eng.capture(decode=True, prefill=False)
    p = g.plan_host.numpy()
    p[0], p[1], p[2] = rows, lens - 1, 1  # the token at position ctx - 1 attends over ctx tokens
    g.plan.copy_(g.plan_host)
    torch.cuda.synchronize()

    def timed(fn, n):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    iters = max(args.steps, 20)
    it_ms = timed(g.graph.replay, iters)
    eng.check_errors()
    # the attention alone, same shapes and metadata: RoPE + KV write and
    # split-K decode of every layer
    cu, ctx, slots, pos, tables = g.meta
    qkv = torch.randn(MODEL_BATCH, cfg.qkv_width, device=device, generator=gen).to(torch.bfloat16)
    cos, sin = eng.runner.cos.index_select(0, pos), eng.runner.sin.index_select(0, pos)
    kc, vc = eng.cache.kv_cache.k_cache, eng.cache.kv_cache.v_cache
    hq, hkv, d = cfg.q_heads, cfg.kv_heads, cfg.head_dim
    q = qkv[:, :hq * d].view(-1, hq, d)
    k = qkv[:, hq * d:(hq + hkv) * d].view(-1, hkv, d)
    v = qkv[:, (hq + hkv) * d:].view(-1, hkv, d)
    q_rot = torch.empty_like(q)
    out = torch.empty_like(q)

    def attention():
        for layer in range(cfg.layers):
            ops.rope_reshape_and_cache(q, k, v, cos, sin, kc, vc, slots, layer, query_out=q_rot, key_out=False)
            ops.paged_decode(q_rot, kc, vc, tables, ctx, layer, out=out, max_context=eng.table_width * BS)

    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        attention()
        torch.cuda.synchronize()
        ga = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ga, stream=stream):
            attention()
    attn_ms = timed(ga.replay, iters)
    ga.reset()
    eng.release()
    kv_bytes = cfg.layers * decode_bytes(lens)
    step_bytes = cfg.weight_bytes() + kv_bytes
    peak, kind = load_peaks()
    gbs = step_bytes / (it_ms * 1e-3) / 1e9
    return {
        "workload": "random-init Qwen2.5-0.5B (24 layers, hidden 896, 14q/2kv, d64, SwiGLU 4864, vocab 151936 tied, "
                    "QKV bias, bf16), 128 sequences, contexts lognormal(median 512, sigma 0.8) clipped [16, 8192], "
                    "shuffled block-16 pool, greedy selection; one step = one captured decode iteration",
        "sequences": MODEL_BATCH, "sum_ctx": int(lens.sum()), "iterations": iters,
        "ms_per_iteration": round(it_ms, 4), "tok_s": round(MODEL_BATCH / (it_ms * 1e-3), 1),
        "attention_ms": round(attn_ms, 4), "attention_share": round(attn_ms / it_ms, 4),
        "weight_mbytes": round(cfg.weight_bytes() / 1e6, 1), "kv_mbytes": round(kv_bytes / 1e6, 1),
        "gbs": round(gbs, 1), "peak_gbs": peak, "peak_kind": kind, "frac": round(gbs / peak, 4),
        "gpu_launches_per_iteration": "pack_step, 3 gathers, 24 x (2 norms, 4 GEMMs, RoPE+write, decode, combine, "
                                      "SiLU*up), lm_head, select, 4 index copies",
    }


# ---------------------------------------------------------------------------
# serving trace: continuous batching, one replica per GPU (config 5)
# ---------------------------------------------------------------------------
SERVE_SEED = 5000
SERVE_RATE_PER_GPU = 3000.0   # arrivals per second per GPU: above what a GPU serves, so the queue never drains
SERVE_WARMUP_STEPS = 150


def run_serving(args, device, world: int, rank: int, group) -> dict:
    """Continuous batching of a Poisson trace, sequence-sharded: the trace's
    requests are placed on the ranks at arrival by ``SequenceDispatcher``
    (fewest reserved tokens, as the free-block rule over a budget that a trace
    never releases), and each rank serves its share with its own replica,
    pool and loop (``ReplicaEngine``: FIFO admission with KV reservations,
    packed prefill, batched decode, greedy selection on the device).  Each
    rank times ``--serve-steps`` engine steps after SERVE_WARMUP_STEPS."""
    from pagedserve_b200.model_runner import QwenConfig, QwenWeights
    from pagedserve_b200.serving import ReplicaEngine, ServeRequest, poisson_trace, prompt_tokens
    from pagedserve_b200.sharding import SequenceDispatcher, gather_counters
    cfg = QwenConfig()
    w = QwenWeights.random(cfg, device, torch.bfloat16, seed=SERVE_SEED)  # the same replica on every rank
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info(device)
    block_bytes = cfg.layers * 2 * cfg.kv_heads * BS * cfg.head_dim * 2
    pool_bytes = min(args.serve_pool_gb * 1e9, free - 24e9)
    nb = int(pool_bytes // block_bytes)
    eng = ReplicaEngine(w, nb, max_running=256, eos_ids=EOS_IDS)
    eng.capture()
    steps = args.serve_steps
    per_rank = 256 + 2 * (SERVE_WARMUP_STEPS + steps)
    trace = poisson_trace(per_rank * world, SERVE_RATE_PER_GPU * world, seed=SERVE_SEED)
    disp = SequenceDispatcher(world, 1 << 50, BS)
    mine = [(i, a, p, o) for i, (a, p, o) in enumerate(trace) if disp.assign(str(i), p + o) == rank]
    nxt = 0
    t0 = time.perf_counter()

    def pump():
        nonlocal nxt
        now = time.perf_counter() - t0
        while nxt < len(mine) and mine[nxt][1] <= now:
            i, a, p, o = mine[nxt]
            eng.submit(ServeRequest(f"t{i}", prompt_tokens(i, p, cfg.vocab, SERVE_SEED), o, arrival=a))
            nxt += 1

    for _ in range(SERVE_WARMUP_STEPS):
        pump()
        eng.step()
    before = dict(eng.stats)
    if group is not None:
        import torch.distributed as dist
        dist.barrier(group=group)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    running = 0
    for _ in range(steps):
        pump()
        eng.step()
        running += len(eng.scheduler.running)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if group is not None:
        import torch.distributed as dist
        dist.barrier(group=group)
    eng.check_errors()
    d = {k: eng.stats[k] - before[k] for k in eng.stats}
    tokens = d["decode_tokens"] + d["first_tokens"]
    mine_stats = {"ms": ms, "tokens": tokens, "decode_tokens": d["decode_tokens"],
                  "first_tokens": d["first_tokens"], "prefill_tokens": d["prefill_tokens"],
                  "finished": d["finished"], "mean_running": running / steps,
                  "queue_left": len(mine) - nxt + len(eng.scheduler.waiting)}
    per = gather_counters(mine_stats, group)
    eng.release()
    del eng
    torch.cuda.empty_cache()
    max_ms = max(r["ms"] for r in per)
    total = sum(r["tokens"] for r in per)
    return {
        "workload": "continuous batching of a Poisson trace (arrivals above service rate), prompts "
                    "lognormal(median 512, sigma 1.0) clipped [16, 8192], outputs geometric(mean 256), contexts "
                    "<= 32768; random-init Qwen2.5-0.5B bf16 replicated per GPU; requests placed on GPUs at arrival "
                    "(SequenceDispatcher); per GPU: FIFO admission with prompt + max_new KV reservations, <= 256 "
                    "running, <= 16384 prefill tokens per step packed into one prefill, one batched decode per step, "
                    "greedy selection + EOS/limit test on the device",
        "pool_gb_per_gpu": round(nb * block_bytes / 1e9, 1), "steps_per_rank": steps,
        "decode_tok_s": round(total / (max_ms * 1e-3), 1),
        "decode_only_tok_s": round(sum(r["decode_tokens"] for r in per) / (max_ms * 1e-3), 1),
        "ms_per_step": round(max_ms / steps, 4),
        "timing": "CUDA events around each rank's timed steps (one host sync per step, so the span includes the "
                  "host loop); aggregate = tokens of all ranks / slowest rank's span",
        "per_rank": [{"tok_s": round(r["tokens"] / (r["ms"] * 1e-3), 1), "ms_per_step": round(r["ms"] / steps, 4),
                      "tokens": int(r["tokens"]), "prefill_tokens": int(r["prefill_tokens"]),
                      "finished": int(r["finished"]), "mean_running": round(r["mean_running"], 1),
                      "queue_left": int(r["queue_left"])} for r in per],
    }


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class Clocks:
    """Samples nvidia-smi clocks/throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = {str(g) for g in gpu_indices}
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or parts[0] not in self.gpus:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (CPU restatement of the reference's algorithm)
# ---------------------------------------------------------------------------
def cpu_oracle_workload(seed: int):
    """The B200 arm's rank-0 decode batch at one GPU (the same 256 context
    lengths, pool size and geometry), with seeded numpy K/V/Q values."""
    from oracle import paged_attention as ora
    rng = np.random.default_rng(seed + 7)
    lens = rank_lengths(1, 0)
    need = int(np.sum(-(-lens // BS)))
    nb = int(math.ceil(SLACK * need))
    perm = rng.permutation(nb)
    tables, at = [], 0
    for n in lens:
        k = -(-int(n) // BS)
        tables.append(perm[at:at + k])
        at += k
    kc = ora.bf16_round(rng.standard_normal((1, nb, HKV, BS, D), dtype=np.float32))
    vc = ora.bf16_round(rng.standard_normal((1, nb, HKV, BS, D), dtype=np.float32))
    q = ora.bf16_round(rng.standard_normal((BATCH, HQ, D), dtype=np.float32))
    new_k = ora.bf16_round(rng.standard_normal((BATCH, HKV, D), dtype=np.float32))
    new_v = ora.bf16_round(rng.standard_normal((BATCH, HKV, D), dtype=np.float32))
    slots = ora.slot_mapping(tables, [int(n) - 1 for n in lens], BS)
    return lens, tables, kc, vc, q, new_k, new_v, slots


def cpu_oracle_call(work, threads: int) -> float:
    """One full 256-sequence decode step of the oracle - each row's new token
    written at its last position, then decode attention over the batch (the
    B200 arm's fused step); returns seconds."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import paged_attention as ora
    lens, tables, kc, vc, q, new_k, new_v, slots = work
    parts = np.array_split(np.arange(BATCH), threads)
    t0 = time.perf_counter()
    ora.reshape_and_cache(new_k, new_v, kc, vc, slots, 0)
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda idx: ora.decode_attention(q[idx], kc, vc, [tables[i] for i in idx], lens[idx], 0),
                    [p for p in parts if len(p)]))
    return time.perf_counter() - t0


def cpu_baseline(seed: int, min_seconds: float = 10.0) -> dict:
    threads = os.cpu_count() or 1
    work = cpu_oracle_workload(seed)
    nbytes = decode_bytes(work[0]) + reshape_bytes(BATCH)
    total, calls = 0.0, 0
    while total < min_seconds and calls < 200:
        total += cpu_oracle_call(work, threads)
        calls += 1
    return {"value": round(nbytes * calls / total / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{calls} full 256-sequence decode steps (new-token write + decode attention) of the numpy "
                      f"oracle (the reference algorithm restated) on the B200 arm's rank-0 context lengths, "
                      f"{total:.1f} s, {threads} threads"}


def workload_config(world: int) -> dict:
    """The headline workload at ``world`` GPUs, from the seeded draws alone
    (both arms report it)."""
    shards = [rank_lengths(world, r) for r in range(world)]
    return {
        "workload": "serving-scale paged decode + reshape_and_cache: 256 x N_gpus requests, ctx lognormal(median "
                    "1024, sigma 0.8) clipped [16, 8192], placed on the GPUs in arrival order by most free KV "
                    "blocks; 14q/2kv heads, d64, block 16, pool 1.25x need per GPU, shuffled blocks",
        "layers": LAYERS, "sequences": int(sum(len(x) for x in shards)),
        "sum_ctx": int(sum(int(x.sum()) for x in shards)),
        "bytes_per_step": int(sum(decode_bytes(x) + reshape_bytes(len(x)) for x in shards)),
        "l2": f"inputs larger than L2: a {LAYERS}-layer pool, consecutive steps are consecutive layers (~180 MB of "
              "KV each, read with an evict-first L2 policy)",
        "launch": f"one CUDA graph per decode iteration: {LAYERS} layer calls, each the fused decode step (new token "
                  "stored through the block table + split-K attention, then the combine), chained by programmatic "
                  "dependent launch; a step is one layer call",
        "parallelism": f"sequence-sharded x{world}",
    }


def run_reference(args, world, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    work = cpu_oracle_workload(WORKLOAD_SEED)
    nbytes = decode_bytes(work[0]) + reshape_bytes(BATCH)
    for _ in range(args.warmup):
        cpu_oracle_call(work, threads)
    t = sum(cpu_oracle_call(work, threads) for _ in range(args.steps))
    value = nbytes * args.steps / t / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * t / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 values, f64 math",
        "data": "synthetic (seeded)",
        "config": workload_config(world),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "per step one full decode step (new-token write + decode attention) over rank "
                                   "0's 256 sequences (the B200 arm's context lengths at one GPU), numpy oracle "
                                   f"(the reference algorithm restated), {threads} host threads"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def build_device_workload(seed: int, device: torch.device, lens: np.ndarray | None = None, layers: int = LAYERS):
    from pagedserve_b200 import PagedKVCache
    rng = np.random.default_rng(seed + 7)
    lens = context_lengths(seed) if lens is None else lens
    batch = len(lens)
    need = int(np.sum(-(-lens // BS)))
    nb = int(math.ceil(SLACK * need))
    cache = PagedKVCache(num_blocks=nb, num_layers=layers, num_kv_heads=HKV, head_dim=D, block_size=BS,
                         dtype=torch.bfloat16, device=device, free_order=rng.permutation(nb))
    ids = [f"seq-{i}" for i in range(batch)]
    for rid, n in zip(ids, lens):
        cache.allocate(rid, int(n))
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    cache.kv_cache.k_cache.normal_(generator=gen)
    cache.kv_cache.v_cache.normal_(generator=gen)
    positions = [int(n) - 1 for n in lens]
    tables = torch.from_numpy(cache.table_rows(ids)).to(device)
    lens_t = torch.from_numpy(lens.astype(np.int32)).to(device)
    slots = torch.tensor([cache.slot_of(r, p) for r, p in zip(ids, positions)], dtype=torch.int64, device=device)
    q = torch.randn(batch, HQ, D, device=device, dtype=torch.bfloat16, generator=gen)
    new_k = torch.randn(batch, HKV, D, device=device, dtype=torch.bfloat16, generator=gen)
    new_v = torch.randn(batch, HKV, D, device=device, dtype=torch.bfloat16, generator=gen)
    return dict(cache=cache, ids=ids, positions=positions, lens=lens, tables=tables, lens_t=lens_t, slots=slots,
                q=q, new_k=new_k, new_v=new_v)


def pin_host_cores(world: int, local: int) -> int:
    """With several ranks on one host, give each its own slice of the allowed
    cores, in order (on a two-socket board the low ranks' GPUs and the low
    cores usually share a socket), so the host-bound end-to-end loops of the
    ranks do not contend or migrate.  Returns the cores this rank keeps."""
    cpus = sorted(os.sched_getaffinity(0))
    per = len(cpus) // max(world, 1)
    if world <= 1 or per < 1:
        return len(cpus)
    os.sched_setaffinity(0, cpus[local * per:(local + 1) * per])
    return per


def run_b200(args, world, rank, local):
    from pagedserve_b200 import ops, paged_decode_attention_with_write
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    host_cores = pin_host_cores(world, local)
    pg, host_group = None, None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # The launcher's process group (NCCL, one rank per GPU) carries no
        # traffic: nothing on the data path crosses GPUs.  Barriers and the
        # end-of-run counters go over a gloo group on host tensors.
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        host_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=300))
        pg = dist
    sections = set(args.sections.split(","))

    LAYERS = args.layers
    w = build_device_workload(WORKLOAD_SEED + rank, device, rank_lengths(world, rank), LAYERS)
    batch = len(w["lens"])
    k, v = w["cache"].kv_cache.k_cache, w["cache"].kv_cache.v_cache
    out = torch.empty_like(w["q"])
    err = torch.zeros(1, dtype=torch.int32, device=device)

    def step(layer):  # the decode step: new token stored + attention, one launch (and the combine)
        ops.paged_decode(w["q"], k, v, w["tables"], w["lens_t"], layer, out=out, error_flag=err,
                         new_key=w["new_k"], new_value=w["new_v"])

    def two_launch(layer):  # the same step as reshape_and_cache, then decode
        ops.reshape_and_cache(w["new_k"], w["new_v"], k, v, w["slots"], layer, error_flag=err)
        ops.paged_decode(w["q"], k, v, w["tables"], w["lens_t"], layer, out=out, error_flag=err)

    def decode_only(layer):
        ops.paged_decode(w["q"], k, v, w["tables"], w["lens_t"], layer, out=out, error_flag=err)

    for layer in range(LAYERS):  # warm the library, size the workspace
        step(layer)
        two_launch(layer)
    torch.cuda.synchronize()

    # One CUDA graph per decode iteration: the 24 layers' decode steps in
    # order, each chained to the one before by programmatic dependent launch.
    # A step is one layer call: K steps are K // 24 iteration graphs plus one
    # graph of the first K % 24 layers.  Graphs of the same shape time the
    # decode kernel alone (for the roofline) and the two-launch form of the
    # step, and one graph per layer call shows the cost of launching each
    # alone.
    stream = torch.cuda.Stream(device)

    def capture(fn, layers):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for layer in layers:
                fn(layer)
        return g

    full, rem = divmod(args.steps, LAYERS)
    graphs = {}
    with torch.cuda.stream(stream):
        for name, fn in (("step", step), ("decode", decode_only), ("two", two_launch)):
            graphs[name] = (capture(fn, range(LAYERS)), capture(fn, range(rem)) if rem else None)
        g_single = [capture(step, [layer]) for layer in range(LAYERS)]
    torch.cuda.synchronize()

    def run_steps(name):
        g_all, g_part = graphs[name]
        for _ in range(full):
            g_all.replay()
        if g_part is not None:
            g_part.replay()

    # Warm every graph the timed region replays, the partial graph of the
    # first K % 24 layers included (its first replay uploads it): at least W
    # warm-up layer calls of each kind.
    for _ in range(-(-args.warmup // LAYERS)):
        for g_all, g_part in graphs.values():
            g_all.replay()
            if g_part is not None:
                g_part.replay()
    for g in g_single:
        g.replay()
    torch.cuda.synchronize()

    def barrier():
        if pg is not None:
            pg.barrier(group=host_group)

    def timed(fn):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        t0.record()
        fn()
        t1.record()
        torch.cuda.synchronize()
        barrier()
        return t0.elapsed_time(t1)

    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_ids = [int(x) for x in visible.split(",")][:max(world, 1)] if visible else list(range(max(world, 1)))
    clocks = Clocks(gpu_ids if rank == 0 else [])
    if rank == 0:
        clocks.__enter__()
    step_ms = timed(lambda: run_steps("step")) / args.steps
    # the decode kernel alone (decode + split-K combine), same K layer calls
    dec_ms = timed(lambda: run_steps("decode")) / args.steps
    # the step as two launches (reshape_and_cache, decode), and one graph launch per layer call
    two_ms = timed(lambda: run_steps("two")) / args.steps
    single_ms = timed(lambda: [g_single[s % LAYERS].replay() for s in range(args.steps)]) / args.steps
    if rank == 0:
        clocks.__exit__(None, None, None)
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag {int(err.item())}")

    # ---- end to end through the reference-facing API, host buffers -------
    # Every step copies its inputs (q, new k, new v: one pinned staging
    # buffer) to the device and its output back to pinned host memory.  Per
    # step s, an upload stream copies step s + 1's inputs and a read-back
    # stream step s - 1's output, both overlapping step s's kernel and each
    # other (PCIe carries both directions at once), as a serving loop
    # pipelines them.  Each step of a run has its own device input buffer and
    # its output is kept until the run ends, so no copy ever waits for a
    # buffer to be free and no memory is reused while a copy reads it.
    cache, ids, positions = w["cache"], w["ids"], w["positions"]
    q_bytes, kv_bytes = w["q"].numel() * 2, w["new_k"].numel() * 2
    in_host = torch.empty(q_bytes + 2 * kv_bytes, dtype=torch.uint8).pin_memory()
    in_host[:q_bytes].view(torch.bfloat16).copy_(w["q"].reshape(-1).cpu())
    in_host[q_bytes:q_bytes + kv_bytes].view(torch.bfloat16).copy_(w["new_k"].reshape(-1).cpu())
    in_host[q_bytes + kv_bytes:].view(torch.bfloat16).copy_(w["new_v"].reshape(-1).cpu())
    e2e_steps = 2 * LAYERS  # timed: two whole decode iterations
    n_buf = e2e_steps + 1
    in_dev = [torch.empty_like(in_host, device=device) for _ in range(n_buf)]
    views = [(buf[:q_bytes].view(torch.bfloat16).view(batch, HQ, 1, D),
              buf[q_bytes:q_bytes + kv_bytes].view(torch.bfloat16).view(batch, HKV, D),
              buf[q_bytes + kv_bytes:].view(torch.bfloat16).view(batch, HKV, D)) for buf in in_dev]
    o_host = [torch.empty((batch, HQ, 1, D), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    s_up, s_down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)
    outs = [None] * n_buf
    # The copies and the events go straight to the CUDA runtime on explicit
    # streams (cuda-python): the same operations as torch's
    # copy_/Event/wait_event, at a fraction of their host cost in this
    # host-bound loop.
    from cuda.bindings import runtime as cudart
    k_h2d, k_d2h = cudart.cudaMemcpyKind.cudaMemcpyHostToDevice, cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost
    rt_ok = cudart.cudaError_t.cudaSuccess

    def rt_check(res):
        if res[0] != rt_ok:
            raise RuntimeError(f"CUDA runtime call failed: {res[0]}")
        return res[1] if len(res) > 1 else None

    def rt_events():
        return [rt_check(cudart.cudaEventCreateWithFlags(cudart.cudaEventDisableTiming)) for _ in range(2)]

    up_h, down_h, comp_h = s_up.cuda_stream, s_down.cuda_stream, compute.cuda_stream
    ev_in, ev_done = rt_events(), rt_events()  # step s's upload / kernel done (slot s % 2)
    in_ptr, in_dev_ptr = in_host.data_ptr(), [b.data_ptr() for b in in_dev]
    in_n, o_n = in_host.numel(), o_host[0].numel() * 2
    o_host_ptr = [t.data_ptr() for t in o_host]

    from pagedserve_b200.attention import clear_metadata_cache

    def upload(s):  # step s's inputs into its own buffer
        rt_check(cudart.cudaMemcpyAsync(in_dev_ptr[s], in_ptr, in_n, k_h2d, up_h))
        rt_check(cudart.cudaEventRecord(ev_in[s % 2], up_h))

    def read_back(s):  # step s's output, once its kernel is done
        rt_check(cudart.cudaStreamWaitEvent(down_h, ev_done[s % 2], 0))
        rt_check(cudart.cudaMemcpyAsync(o_host_ptr[s % 2], outs[s].data_ptr(), o_n, k_d2h, down_h))

    # Each decode iteration passes new positions, as a serving loop does: here
    # iteration k decodes at positions ctx - 1 - k (inside each request's
    # reserved capacity), so its first layer call rebuilds and copies the
    # lengths; the block table stays on the device while the cache epoch and
    # the request list do not change.
    iter_positions = [[p - k for p in positions] for k in range(4)]
    host_us = [0.0, 0.0]  # host time in the API call: first layer call of an iteration, the others

    def e2e_step(s, first_iteration):
        layer = s % LAYERS
        pos = iter_positions[first_iteration + s // LAYERS]
        if s >= 1:
            read_back(s - 1)
        upload(s + 1)
        rt_check(cudart.cudaStreamWaitEvent(comp_h, ev_in[s % 2], 0))
        qd, kd, vd = views[s]
        h0 = time.perf_counter()
        outs[s] = paged_decode_attention_with_write(qd, kd, vd, cache, ids, pos, layer)
        host_us[0 if layer == 0 else 1] += 1e6 * (time.perf_counter() - h0)
        rt_check(cudart.cudaEventRecord(ev_done[s % 2], comp_h))

    def e2e_run(n, first_iteration):
        s_up.wait_stream(compute)
        s_down.wait_stream(compute)
        upload(0)
        for s in range(n):
            e2e_step(s, first_iteration)
        read_back(n - 1)
        compute.wait_stream(s_up)
        compute.wait_stream(s_down)

    # as many warm-up steps as timed ones (pinned staging, the metadata path
    # and the allocator's cached blocks for the outputs all warm), then whole
    # iterations timed: every iteration's first layer call rebuilds and copies
    # the lengths, as a new iteration would
    clear_metadata_cache(cache)
    e2e_run(e2e_steps, 0)
    torch.cuda.synchronize()
    outs[:] = [None] * n_buf  # back to the allocator, which hands them to the timed steps
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    host_us[:] = [0.0, 0.0]
    h_start = time.perf_counter()
    e_start.record(compute)
    e2e_run(e2e_steps, e2e_steps // LAYERS)
    e_end.record(compute)
    host_loop_us = 1e6 * (time.perf_counter() - h_start) / e2e_steps
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e_start.elapsed_time(e_end) / e2e_steps
    for ev in ev_in + ev_done:
        rt_check(cudart.cudaEventDestroy(ev))
    outs[:] = [None] * n_buf
    iterations = e2e_steps // LAYERS  # lengths copies inside the timed region
    h2d = in_host.numel() + 4 * batch * iterations / e2e_steps
    # iteration k attends over ctx - k tokens per request
    e2e_rank_bytes = sum(decode_bytes(w["lens"] - k) + reshape_bytes(batch) for k in range(1, 1 + iterations)) / iterations
    d2h = o_host[0].numel() * 2

    # ---- reduce over ranks (gloo, host tensors): times by max, work by sum ----
    from pagedserve_b200.sharding import gather_counters
    lens = w["lens"]
    step_bytes = decode_bytes(lens) + reshape_bytes(batch)
    rank_step_ms = step_ms
    per_rank = gather_counters({"step_ms": step_ms, "dec_ms": dec_ms, "e2e_ms": e2e_ms, "e2e_host_us": host_loop_us,
                                "host_cores": host_cores, "single_ms": single_ms,
                                "two_ms": two_ms, "bytes": step_bytes, "e2e_bytes": e2e_rank_bytes, "seqs": batch,
                                "ctx": int(lens.sum())}, host_group)
    step_ms, dec_ms, e2e_ms, single_ms, two_ms = (max(r[k] for r in per_rank) for k in
                                                 ("step_ms", "dec_ms", "e2e_ms", "single_ms", "two_ms"))
    total_bytes, total_seqs = sum(r["bytes"] for r in per_rank), int(sum(r["seqs"] for r in per_rank))
    del w, graphs, g_single, in_dev, views, outs
    torch.cuda.empty_cache()

    # ---- the other sections (each rank on its own GPU) ----------------------
    prefill = run_prefill(args, device, 2000 + rank) if "prefill" in sections else None
    select = run_select(args, device, 3000 + rank) if "select" in sections else None
    model = run_model_decode(args, device, 4000) if "model" in sections else None
    torch.cuda.empty_cache()
    serving = run_serving(args, device, world, rank, host_group) if "serve" in sections else None
    value = total_bytes / (step_ms * 1e-3) / 1e9
    e2e_value = sum(r["e2e_bytes"] for r in per_rank) / (e2e_ms * 1e-3) / 1e9
    peak, peak_kind = load_peaks()
    achieved = step_bytes / (rank_step_ms * 1e-3) / 1e9

    if rank == 0:
        cpu = cpu_baseline(WORKLOAD_SEED) if world == 1 else None
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) KV/Q, lognormal contexts)",
            "config": workload_config(world),
            "detail": {
                "per_layer_graph_ms": round(single_ms, 5),
                "per_layer_graph_note": "the same layer calls launched as one CUDA graph each",
                "two_launch_ms": round(two_ms, 5),
                "two_launch_note": "the step as reshape_and_cache (slot mapping) then decode, same graphs",
                "per_rank": [{"step_ms": round(r["step_ms"], 5), "sequences": int(r["seqs"]), "sum_ctx": int(r["ctx"]),
                              "gbs": round(r["bytes"] / (r["step_ms"] * 1e-3) / 1e9, 1),
                              "e2e_ms": round(r["e2e_ms"], 5), "e2e_host_us_per_step": round(r["e2e_host_us"], 1),
                              "host_cores": int(r["host_cores"])} for r in per_rank],
            },
            "pct_of_8tbs": round(100 * value / world / NOMINAL_HBM_GBS, 2),
            "pct_of_measured_peak": round(100 * value / world / peak, 2),
            "attn_layer_tok_per_s": round(total_seqs / (step_ms * 1e-3), 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "kernel": "decode_fast_kernel<bf16, 2, append> + decode_combine_kernel (the fused step)",
                         "timing": "CUDA events around the K layer calls (iteration graphs) on this rank; average "
                                   "per layer call",
                         "bytes_per_launch": step_bytes,
                         "avg_launch_ms": round(rank_step_ms, 5), "traffic": STEP_TRAFFIC_BYTES,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one fused decode "
                                           "and one combine launch on this seeded workload (decode ncu summary "
                                           "under profiles/)",
                         "decode_only_ms": round(dec_ms, 5),
                         "decode_only_note": "decode + combine without the new-token store, same graphs"},
            "e2e": {"value": round(e2e_value, 3), "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": round(e2e_ms, 4), "steps": e2e_steps,
                    "host_us_per_step": round(host_loop_us, 1),
                    "api_host_us": {"first_call_of_iteration": round(host_us[0] / (e2e_steps // LAYERS), 1),
                                    "other_calls": round(host_us[1] / (e2e_steps - e2e_steps // LAYERS), 1)},
                    "path": "per layer call: q, new k, new v copied from one pinned host staging buffer, "
                            "paged_decode_attention_with_write (reference-facing API: write_token + decode in "
                            "one launch), output copied back to pinned host memory; the upload of step s + 1 "
                            "(a device input buffer per step, outputs kept until the run ends) and the read-back "
                            "of step s - 1 on two copy streams (cudaMemcpyAsync), overlapping step s's kernel and "
                            "each other; each iteration's first layer call rebuilds and "
                            "copies the lengths for its new positions (the block table stays on the device within "
                            f"a cache epoch); timed over 2 whole iterations ({LAYERS} layer calls each) after two "
                            "of warm-up"},
            "gpu_launches": 2 * args.steps,
            "gpu_launches_note": "per step: decode (with the new-token store), combine",
            "clocks": clocks.summary(),
            "decode": model,
            "serving": serving,
            "prefill": prefill,
            "select_tokens": select,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--serve-steps", type=int, default=600,
                    help="engine steps each rank times in the serving trace")
    ap.add_argument("--serve-pool-gb", type=float, default=150.0,
                    help="KV pool per GPU for the serving trace (capped by free memory)")
    ap.add_argument("--sections", default="decode,prefill,select,model,serve",
                    help="comma-separated sections besides the headline decode step")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers in the pool and the iteration graph (default: the model's 24); every step is "
                         "still one full layer call, so fewer only shrink the device memory a profiler must "
                         "save and restore")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.layers < 2:
        ap.error("--layers must be at least 2 (consecutive steps must not reuse one layer's KV from L2)")
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_b200(args, world, rank, local)


if __name__ == "__main__":
    main()
