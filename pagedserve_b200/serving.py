"""One GPU's serving loop: FIFO admission, packed prefill, batched decode.

The reference serves through ``ContinuousBatcher._run``
(pagedserve/engine/continuous_batcher.py:132-417) on one device:

* ``Scheduler.schedule`` admits waiting requests in strict FIFO order while
  fewer than ``max_running_requests`` run and the queue head's KV reservation
  (prompt + max_new_tokens, in blocks) fits (pagedserve/engine/scheduler.py:68-109);
* every admitted request is prefilled on its own through
  ``_forward_paged`` and its first token taken with ``.item()``
  (continuous_batcher.py:268-295);
* every running request then decodes one token in ONE batched forward
  (``_forward_paged_batch``), followed by a per-row ``.item()`` /
  ``add_generated_token`` / EOS loop (continuous_batcher.py:302-364).

``ReplicaEngine.step`` keeps that order and those rules, and runs each half
as one captured CUDA graph on this package's kernels:

* the step's admitted prompts are packed into one prefill (``PrefillGraph``:
  ``pack_step`` builds cu_seqlens, slots and positions on the device, then
  ``PagedModelRunner.prefill`` and ``select_tokens``);
* the decode is one ``DecodeGraph`` replay (``pack_step``, the 24-layer
  decode, ``lm_head``, ``select_tokens``), with each request's last token and
  remaining-token counter kept on the device, indexed by its row in the
  block-table store, so nothing but the step plan crosses PCIe on the way in
  and only the tokens and status bytes on the way out.

Graphs are captured for a few batch-size and token-count buckets; rows and
tokens past the step's real ones are padding that runs against one reserved
"pad" request (its K/V writes go to its own blocks, its outputs are
ignored).  One process per GPU runs one engine over its own pool; requests
are placed on GPUs before they arrive (``sharding.SequenceDispatcher``), so
the engines never talk to each other.
"""

from __future__ import annotations

import bisect
import dataclasses
import math
from collections import deque

import numpy as np
import torch

from . import ops
from .model_runner import PagedModelRunner, QwenConfig, QwenWeights
from .paged_kv import PagedKVCache

PAD_REQUEST = "__pad__"
PAD_TOKENS = 128          # the pad request's capacity: padding sequences are at most this long
_BIG_REMAINING = 1 << 30  # the pad row never reaches a generation limit


@dataclasses.dataclass
class ServeRequest:
    """A request as the scheduler sees it (pagedserve/engine/request.py:40-86):
    prompt, generation budget, tokens generated so far, state."""

    request_id: str
    prompt_token_ids: np.ndarray
    max_new_tokens: int
    arrival: float = 0.0
    generated: int = 0
    finished: bool = False
    eos: bool = False
    tokens: list | None = None  # generated ids, when the engine records them

    @property
    def num_prompt_tokens(self) -> int:
        return int(len(self.prompt_token_ids))

    @property
    def capacity(self) -> int:
        """KV tokens reserved at admission (scheduler.py:82-86)."""
        return self.num_prompt_tokens + self.max_new_tokens

    @property
    def position(self) -> int:
        """Position of the token the next decode step feeds
        (continuous_batcher.py:316-319: num_prompt + num_generated - 1)."""
        return self.num_prompt_tokens + self.generated - 1


class FifoScheduler:
    """Strict-FIFO admission with a KV reservation per request, as
    ``Scheduler.schedule`` (scheduler.py:68-109): the queue head is admitted
    while fewer than ``max_running`` requests run and its prompt +
    max_new_tokens blocks are free; a head that does not fit blocks the
    queue.  One addition for the packed prefill: a step admits at most
    ``max_prefill_tokens`` prompt tokens and ``max_prefill_seqs`` requests
    (the rest wait for the next step, still in order)."""

    def __init__(self, cache: PagedKVCache, max_running: int, max_prefill_tokens: int, max_prefill_seqs: int):
        if max_running <= 0:
            raise ValueError("max_running_requests must be positive")
        self.cache = cache
        self.max_running = max_running
        self.max_prefill_tokens = max_prefill_tokens
        self.max_prefill_seqs = max_prefill_seqs
        self.waiting: deque[ServeRequest] = deque()
        self.running: dict[str, ServeRequest] = {}

    def submit(self, req: ServeRequest) -> None:
        if req.request_id in self.running or req.request_id == PAD_REQUEST:
            raise ValueError(f"Duplicate request ID: {req.request_id!r}")
        if req.num_prompt_tokens == 0:
            raise ValueError("prompt_token_ids cannot be empty")
        if req.num_prompt_tokens > self.max_prefill_tokens:
            raise ValueError(f"prompt of {req.num_prompt_tokens} tokens exceeds the prefill budget "
                             f"({self.max_prefill_tokens})")
        self.waiting.append(req)

    def schedule(self) -> list[ServeRequest]:
        admitted, tokens = [], 0
        while self.waiting and len(self.running) < self.max_running and len(admitted) < self.max_prefill_seqs:
            req = self.waiting[0]
            if tokens + req.num_prompt_tokens > self.max_prefill_tokens:
                break
            if self.cache.block_manager.blocks_needed(req.capacity) > self.cache.free_blocks:
                break  # strict FIFO: the head is not skipped
            self.cache.allocate(req.request_id, req.capacity)
            self.waiting.popleft()
            self.running[req.request_id] = req
            admitted.append(req)
            tokens += req.num_prompt_tokens
        return admitted

    def complete(self, request_id: str) -> ServeRequest:
        req = self.running.pop(request_id)
        self.cache.free(request_id)
        req.finished = True
        return req


def _bucket(buckets: list[int], n: int) -> int:
    i = bisect.bisect_left(buckets, n)
    if i == len(buckets):
        raise ValueError(f"{n} exceeds the largest captured bucket ({buckets[-1]})")
    return buckets[i]


class _StepGraph:
    """Static buffers + one captured step.

    A decode step has ``entries`` decode rows.  A mixed step has
    ``prefill_entries`` prompt entries (admitted prompts, then pad sequences
    filling ``prefill_tokens``) followed by ``entries - prefill_entries``
    decode rows; its tokens are the prompt tokens then one per decode row.
    The plan rows (device int32) are [store row, first new position, new
    tokens, generation budget] per entry (the budget is read for prompt
    entries only; decode rows keep theirs on the device)."""

    def __init__(self, engine: "ReplicaEngine", entries: int, prefill_entries: int = 0, prefill_tokens: int = 0):
        dev = engine.device
        self.entries, self.prefill_entries, self.prefill_tokens = entries, prefill_entries, prefill_tokens
        self.decode_rows = entries - prefill_entries
        self.tokens = prefill_tokens + self.decode_rows
        self.mixed = prefill_entries > 0
        self.plan_host = torch.zeros((4, entries), dtype=torch.int32).pin_memory()
        self.plan = torch.zeros((4, entries), dtype=torch.int32, device=dev)
        self.tok_host = torch.zeros(max(prefill_tokens, 1), dtype=torch.int64).pin_memory() if self.mixed else None
        self.tok_in = torch.zeros(self.tokens, dtype=torch.int64, device=dev) if self.mixed else None
        w = engine.table_width
        self.meta = (torch.zeros(entries + 1, dtype=torch.int32, device=dev),
                     torch.zeros(entries, dtype=torch.int32, device=dev),
                     torch.zeros(self.tokens, dtype=torch.int64, device=dev),
                     torch.zeros(self.tokens, dtype=torch.int64, device=dev),
                     torch.zeros((entries, w), dtype=torch.int32, device=dev))
        # rows of the logits: each prompt entry's last token, then every decode row
        self.decode_last = torch.arange(prefill_tokens, self.tokens, dtype=torch.int64, device=dev)
        self.tok_out = torch.zeros(entries, dtype=torch.int64, device=dev)
        self.status = torch.zeros(entries, dtype=torch.uint8, device=dev)
        self.out_host = torch.zeros(entries * 9, dtype=torch.uint8).pin_memory()
        self.graph: torch.cuda.CUDAGraph | None = None

    def body(self, e: "ReplicaEngine") -> None:
        plan = self.plan
        ops.pack_step(e.table_store, plan[0], plan[1], plan[2], self.tokens, e.block_size, e.table_width,
                      error_flag=e.err, out=self.meta)
        cu, ctx, slots, pos, tables = self.meta
        rows = plan[0].long()
        rem = e.remaining.index_select(0, rows)
        max_context = e.table_width * e.block_size
        if self.mixed:
            ep = self.prefill_entries
            rem[:ep].copy_(plan[3][:ep])  # the admitted requests' budgets
            self.tok_in[self.prefill_tokens:].copy_(e.last_token.index_select(0, rows[ep:]))
            last = torch.cat([(cu[1:ep + 1] - 1).clamp_(min=0).long(), self.decode_last])
            logits = e.runner.mixed(self.tok_in, pos, slots, self.prefill_tokens, cu[:ep + 1], e.max_prompt,
                                    tables[ep:], ctx[ep:], last, max_context=max_context)
        else:
            tokens_in = e.last_token.index_select(0, rows)
            logits = e.runner.decode(tokens_in, pos, tables, ctx, slots, max_context=max_context)
        ops.select_tokens(logits, e.eos, rem, tokens=self.tok_out, status=self.status, error_flag=e.err)
        e.last_token.index_copy_(0, rows, self.tok_out)
        e.remaining.index_copy_(0, rows, rem)

    def capture(self, e: "ReplicaEngine") -> None:
        s = torch.cuda.Stream(e.device)
        s.wait_stream(torch.cuda.current_stream(e.device))
        with torch.cuda.stream(s):
            self.body(e)  # warm-up run: cuBLAS handles, library workspaces
        torch.cuda.current_stream(e.device).wait_stream(s)
        torch.cuda.synchronize(e.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=e.graph_pool):
            self.body(e)
        torch.cuda.synchronize(e.device)

    def run(self, e: "ReplicaEngine") -> tuple[np.ndarray, np.ndarray]:
        """Upload the plan (and prompt tokens), replay, read tokens and status back."""
        stream = torch.cuda.current_stream(e.device)
        self.plan.copy_(self.plan_host, non_blocking=True)
        if self.mixed:
            self.tok_in[: self.prefill_tokens].copy_(self.tok_host[: self.prefill_tokens], non_blocking=True)
        self.graph.replay()
        n = self.entries
        out = self.out_host
        out[: 8 * n].view(torch.int64).copy_(self.tok_out, non_blocking=True)
        out[8 * n:].copy_(self.status, non_blocking=True)
        stream.synchronize()
        return out[: 8 * n].view(torch.int64).numpy(), out[8 * n:].numpy()


class ReplicaEngine:
    """A model replica, its KV pool and its serving loop on one GPU."""

    def __init__(self, weights: QwenWeights, num_blocks: int, *, block_size: int = 16, max_running: int = 256,
                 max_prefill_tokens: int = 16384, max_prefill_seqs: int = 32, max_prompt: int = 8192,
                 max_context: int = 32768, eos_ids=(), decode_buckets=(64, 128, 256),
                 prefill_buckets=(256, 512, 1024, 1536, 2048, 3072, 4096, 6144, 8192, 12288, 16384),
                 record_tokens: bool = False, free_order=None):
        cfg: QwenConfig = weights.cfg
        self.cfg, self.device = cfg, weights.device
        self.block_size = block_size
        self.max_prompt = max_prompt
        self.table_width = -(-max_context // block_size)
        self.cache = PagedKVCache(num_blocks=num_blocks, num_layers=cfg.layers, num_kv_heads=cfg.kv_heads,
                                  head_dim=cfg.head_dim, block_size=block_size, dtype=weights.dtype,
                                  device=self.device, free_order=free_order)
        self.runner = PagedModelRunner(weights, self.cache.kv_cache.k_cache, self.cache.kv_cache.v_cache, block_size)
        self.scheduler = FifoScheduler(self.cache, max_running, max_prefill_tokens, max_prefill_seqs)
        self.record_tokens = record_tokens
        rows = max_running + 2
        dev = self.device
        self.table_store = torch.zeros((rows, self.table_width), dtype=torch.int32, device=dev)
        self.last_token = torch.zeros(rows, dtype=torch.int64, device=dev)
        self.remaining = torch.zeros(rows, dtype=torch.int32, device=dev)
        self.eos = torch.tensor(sorted({int(e) for e in eos_ids}), dtype=torch.int64, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        # the pad request: padding rows and tokens of captured steps run against it
        self.cache.allocate(PAD_REQUEST, PAD_TOKENS)
        self.pad_row = self._store_row(PAD_REQUEST)
        self._upload_tables([PAD_REQUEST])
        self.remaining[self.pad_row] = _BIG_REMAINING
        self.graph_pool = torch.cuda.graph_pool_handle()
        self.decode_buckets = sorted(b for b in decode_buckets if b <= max_running) or [max_running]
        if self.decode_buckets[-1] < max_running:
            self.decode_buckets.append(max_running)
        self.prefill_buckets = sorted(prefill_buckets)
        if self.prefill_buckets[-1] < max_prefill_tokens:
            raise ValueError("the largest prefill bucket must hold max_prefill_tokens")
        self._decode = {b: _StepGraph(self, b) for b in self.decode_buckets}
        # a step with admissions: its prompts (padded to the bucket) and up to
        # max_running decode rows in one pass
        self._mixed = {t: _StepGraph(self, max_prefill_seqs + -(-t // PAD_TOKENS) + max_running,
                                     max_prefill_seqs + -(-t // PAD_TOKENS), t)
                       for t in self.prefill_buckets}
        # per store row: the request there, its prompt length, tokens generated, decoding or not
        self._req_by_row: list[ServeRequest | None] = [None] * rows
        self._prompt_len = np.zeros(rows, dtype=np.int32)
        self._generated = np.zeros(rows, dtype=np.int32)
        self._decoding = np.zeros(rows, dtype=bool)
        self.stats = dict(steps=0, decode_steps=0, prefill_steps=0, decode_tokens=0, prefill_tokens=0,
                          first_tokens=0, finished=0, decode_rows=0)

    # -- set-up ---------------------------------------------------------------
    def capture(self, decode: bool = True, prefill: bool = True) -> None:
        """Capture every bucket's graph (before serving; the first replay of
        each would otherwise pay for it)."""
        graphs = (list(self._decode.values()) if decode else []) + (list(self._mixed.values()) if prefill else [])
        for g in graphs:
            self._fill_pad_plan(g)
            g.plan.copy_(g.plan_host)
            g.capture(self)
        self.remaining[self.pad_row] = _BIG_REMAINING

    def release(self) -> None:
        for g in list(self._decode.values()) + list(self._mixed.values()):
            if g.graph is not None:
                g.graph.reset()
                g.graph = None

    def _store_row(self, request_id: str) -> int:
        row = self.cache.get_block_table(request_id)._row
        if not 0 <= row < self.table_store.shape[0]:
            raise RuntimeError("table-store row out of range")
        return row

    def _upload_tables(self, request_ids) -> None:
        rows = [self._store_row(r) for r in request_ids]
        host = torch.from_numpy(self.cache.table_rows(request_ids, width=self.table_width)).pin_memory()
        dev = host.to(self.device, non_blocking=True)
        self.table_store.index_copy_(0, torch.tensor(rows, dtype=torch.int64).to(self.device, non_blocking=True), dev)

    def _pad_decode(self, p: np.ndarray, first: int, last: int) -> None:
        """Decode entries ``first .. last - 1`` that carry no request: one
        token of the pad request at position 0."""
        p[0, first:last] = self.pad_row
        p[1, first:last] = 0
        p[2, first:last] = 1
        p[3, first:last] = _BIG_REMAINING

    def _pad_prefill(self, p: np.ndarray, g: _StepGraph, used_entries: int, used_tokens: int) -> None:
        """Prompt entries past the admitted ones: the bucket's spare tokens as
        pad-request sequences of at most PAD_TOKENS tokens, then empty ones."""
        ep = g.prefill_entries
        p[0, used_entries:ep] = self.pad_row
        p[1, used_entries:ep] = 0
        p[2, used_entries:ep] = 0
        p[3, used_entries:ep] = _BIG_REMAINING
        spare, e = g.prefill_tokens - used_tokens, used_entries
        while spare > 0:
            n = min(spare, PAD_TOKENS)
            p[2, e] = n
            spare -= n
            e += 1

    def _fill_pad_plan(self, g: _StepGraph) -> None:
        """A plan of padding only (for the capture's warm-up run)."""
        p = g.plan_host.numpy()
        if g.mixed:
            self._pad_prefill(p, g, 0, 0)
        self._pad_decode(p, g.prefill_entries, g.entries)

    # -- serving ----------------------------------------------------------------
    def submit(self, req: ServeRequest) -> None:
        self.scheduler.submit(req)

    @property
    def has_work(self) -> bool:
        return bool(self.scheduler.waiting or self.scheduler.running)

    def step(self) -> list[ServeRequest]:
        """Admit, then one pass for every running request: the admitted
        prompts prefilled (packed) and every request already decoding one
        token, in the same launches.  Returns the requests that finished.

        The reference prefills the admitted requests and then decodes every
        running one, a new request taking its first decode token in the same
        iteration (continuous_batcher.py:261-364); here a new request takes
        its first (prefill) token this step and decodes from the next, so
        every request's token sequence is the same."""
        admitted = self.scheduler.schedule()
        rows = np.flatnonzero(self._decoding).astype(np.int32)
        if admitted:
            finished = self._mixed_step(admitted, rows)
        elif rows.size:
            finished = self._decode_step(rows)
        else:
            finished = []
        self.stats["steps"] += 1
        return finished

    def _decode_plan(self, p: np.ndarray, at: int, rows: np.ndarray) -> None:
        n = rows.size
        p[0, at:at + n] = rows
        # the token fed sits at num_prompt + num_generated - 1 (continuous_batcher.py:316-319)
        p[1, at:at + n] = self._prompt_len[rows] + self._generated[rows] - 1
        p[2, at:at + n] = 1

    def _mixed_step(self, admitted: list[ServeRequest], rows_dec: np.ndarray) -> list[ServeRequest]:
        ids = [r.request_id for r in admitted]
        self._upload_tables(ids)
        total = sum(r.num_prompt_tokens for r in admitted)
        g = self._mixed[_bucket(self.prefill_buckets, total)]
        if rows_dec.size > g.decode_rows:
            raise RuntimeError("more decode rows than the step graph holds")
        p = g.plan_host.numpy()
        toks = g.tok_host.numpy()
        rows = np.empty(len(admitted), dtype=np.int32)
        at = 0
        for i, r in enumerate(admitted):
            n = r.num_prompt_tokens
            row = self._store_row(r.request_id)
            rows[i] = row
            self._req_by_row[row] = r
            self._prompt_len[row] = n
            self._generated[row] = 0
            p[0, i], p[1, i], p[2, i], p[3, i] = row, 0, n, r.max_new_tokens
            toks[at:at + n] = r.prompt_token_ids
            at += n
        toks[at:g.prefill_tokens] = 0
        self._pad_prefill(p, g, len(admitted), total)
        ep = g.prefill_entries
        self._decode_plan(p, ep, rows_dec)
        self._pad_decode(p, ep + rows_dec.size, g.entries)
        tokens, status = g.run(self)
        self.stats["prefill_steps"] += 1
        self.stats["prefill_tokens"] += total
        self.stats["first_tokens"] += len(admitted)
        self.stats["decode_steps"] += 1 if rows_dec.size else 0
        self.stats["decode_tokens"] += rows_dec.size
        self.stats["decode_rows"] += g.decode_rows
        self._decoding[rows] = True
        done = self._apply(rows, tokens[: len(admitted)], status[: len(admitted)])
        if rows_dec.size:
            done += self._apply(rows_dec, tokens[ep:ep + rows_dec.size], status[ep:ep + rows_dec.size])
        return done

    def _decode_step(self, rows: np.ndarray) -> list[ServeRequest]:
        n = rows.size
        g = self._decode[_bucket(self.decode_buckets, n)]
        p = g.plan_host.numpy()
        self._decode_plan(p, 0, rows)
        self._pad_decode(p, n, g.entries)
        tokens, status = g.run(self)
        self.stats["decode_steps"] += 1
        self.stats["decode_tokens"] += n
        self.stats["decode_rows"] += g.entries
        return self._apply(rows, tokens, status)

    def _apply(self, rows: np.ndarray, tokens: np.ndarray, status: np.ndarray) -> list[ServeRequest]:
        """The reference's per-row loop (continuous_batcher.py:333-360) over
        the step's host copy: count the token, finish on EOS or on the last
        allowed token (``status``: the device's finish test)."""
        n = rows.size
        st = status[:n]
        if np.any(st & ops.SELECT_LIMIT):
            raise RuntimeError("Request has reached its generation limit")
        self._generated[rows] += 1
        if self.record_tokens:
            for i, row in enumerate(rows):
                r = self._req_by_row[row]
                if r.tokens is None:
                    r.tokens = []
                r.tokens.append(int(tokens[i]))
        done = []
        for i in np.flatnonzero(st & ops.SELECT_DONE):
            row = int(rows[i])
            r = self._req_by_row[row]
            r.generated = int(self._generated[row])
            r.eos = bool(st[i] & ops.SELECT_EOS)
            self._decoding[row] = False
            self._req_by_row[row] = None
            self.scheduler.complete(r.request_id)
            done.append(r)
        self.stats["finished"] += len(done)
        return done

    def check_errors(self) -> None:
        bits = int(self.err.item())
        if bits:
            from ._native import describe_device_error
            raise RuntimeError(f"device error flag {bits}: {describe_device_error(bits)}")


def poisson_trace(n: int, rate: float, seed: int, prompt_median: float = 512, prompt_sigma: float = 1.0,
                  prompt_lo: int = 16, prompt_hi: int = 8192, output_mean: float = 256, max_context: int = 32768
                  ) -> list[tuple[float, int, int]]:
    """``n`` requests as (arrival seconds, prompt tokens, max new tokens):
    Poisson arrivals at ``rate`` per second, prompt lengths lognormal
    (``prompt_median``, ``prompt_sigma``) clipped to [lo, hi], output
    lengths geometric with mean ``output_mean``, prompt + output <= max_context."""
    rng = np.random.default_rng(seed)
    arrivals = np.cumsum(rng.exponential(1.0 / rate, n))
    prompts = np.clip(np.round(rng.lognormal(math.log(prompt_median), prompt_sigma, n)), prompt_lo, prompt_hi)
    outputs = rng.geometric(1.0 / output_mean, n)
    outputs = np.minimum(outputs, max_context - prompts)
    return [(float(a), int(p), int(o)) for a, p, o in zip(arrivals, prompts, outputs)]


def prompt_tokens(index: int, length: int, vocab: int, seed: int) -> np.ndarray:
    """Synthetic prompt ids of request ``index`` (seeded, uniform over the vocabulary)."""
    return np.random.default_rng((seed, index)).integers(0, vocab, length, dtype=np.int64)
