"""Device-side greedy selection (psb_select_tokens) against the reference's
own argmax + Request bookkeeping (golden vectors), the oracle, and
torch.argmax on the device, from single rows to the serving batch over the
full Qwen2.5 vocabulary."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import select_tokens as sel
from tests.helpers import TORCH_DTYPES

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "select_outputs.npz"))
VOCAB = 151936
DTYPE_OF = {"bf16": "bfloat16", "f16": "float16", "f32": "float32", "bf16_ties": "bfloat16"}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import pagedserve_b200._native as native
    native.load()


def _run(logits, eos, remaining, ctas=0):
    from pagedserve_b200 import ops
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rem = remaining.clone()
    tokens, status = ops.select_tokens(logits, eos, rem, error_flag=err, ctas_per_row=ctas)
    torch.cuda.synchronize()
    return tokens.cpu().numpy(), status.cpu().numpy(), rem.cpu().numpy(), int(err.item())


@pytest.mark.parametrize("name", ["bf16", "f16", "f32", "bf16_ties"])
@pytest.mark.parametrize("ctas", [0, 1, 3, 8])
def test_matches_reference_selection(name, ctas):
    """[B, S, V] logits as the model returns them; the last position is used."""
    logits = torch.from_numpy(GOLD[f"{name}/logits"]).cuda().to(TORCH_DTYPES[DTYPE_OF[name]])
    eos = torch.from_numpy(GOLD["eos_ids"]).cuda()
    rem = torch.from_numpy(GOLD[f"{name}/remaining"]).cuda()
    tokens, status, rem_after, err = _run(logits, eos, rem, ctas)
    assert np.array_equal(tokens, GOLD[f"{name}/tokens"])
    assert np.array_equal(status, GOLD[f"{name}/status"])
    assert np.array_equal(rem_after, GOLD[f"{name}/remaining_after"])
    assert bool(err & 64) == bool(np.any(GOLD[f"{name}/status"] & sel.LIMIT))


def _edge_batch(b, v, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (4.0 * torch.randn(b, v, generator=g, device="cuda")).to(TORCH_DTYPES[dtype])
    if b >= 8:
        x[0] = float("-inf")
        x[1, [v - 1, v // 3]] = float("nan")
        x[2] = 0.0
        x[2, : v // 2] = -0.0
        x[3, [v // 2, v - 1]] = float("inf")
        x[4] = 1.0
        x[5, v - 1] = 1e4
        x[6] = torch.round(x[6])
        x[7, 0] = float("nan")
    return x


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("b,v", [(1, 1), (3, 7), (9, 33), (16, 1000), (8, 4099), (64, VOCAB)])
def test_matches_torch_argmax_and_oracle(dtype, b, v):
    x = _edge_batch(b, v, dtype, b * 1000 + v)
    eos = torch.tensor([0, 5], dtype=torch.int64, device="cuda")
    rem = torch.full((b,), 4, dtype=torch.int32, device="cuda")
    for ctas in (0, 1, 2, 5, 8):
        tokens, status, rem_after, err = _run(x, eos, rem, ctas)
        assert np.array_equal(tokens, x.argmax(dim=-1).cpu().numpy()), ctas
        t2, s2, r2, limit = sel.select_tokens(x.float().cpu().numpy(), [0, 5], rem.cpu().numpy())
        assert np.array_equal(tokens, t2) and np.array_equal(status, s2) and np.array_equal(rem_after, r2)
        assert err == 0 and not limit


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_strided_and_unaligned_rows(dtype):
    """A [B, S, V] view's last position (row stride S*V) and rows that start
    off a 16-byte boundary (the element-wise path)."""
    b, s, v = 12, 3, 5003
    x = _edge_batch(b * s, v, dtype, 7).view(b, s, v)
    eos = torch.tensor([], dtype=torch.int64, device="cuda")
    rem = torch.full((b,), 9, dtype=torch.int32, device="cuda")
    tokens, status, _, _ = _run(x, eos, rem)
    assert np.array_equal(tokens, x[:, -1, :].argmax(dim=-1).cpu().numpy())
    assert not status.any()
    flat = _edge_batch(b, v + 1, dtype, 8)
    shifted = flat[:, 1:]  # base off the 16-byte boundary, stride v + 1
    tokens, _, _, _ = _run(shifted, eos, rem)
    assert np.array_equal(tokens, shifted.argmax(dim=-1).cpu().numpy())


def test_serving_batch_full_vocab_with_stops():
    """The decode batch of the serving workload over the full vocabulary: EOS
    hits, last allowed tokens, and rows already at their limit."""
    b = 256
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(b, VOCAB, generator=g, device="cuda").to(torch.bfloat16)
    eos = torch.tensor([151643, 151645], dtype=torch.int64, device="cuda")
    x[10, 151643] = 100.0
    x[11, 151645] = 100.0
    rem_np = np.random.default_rng(4).integers(1, 50, b).astype(np.int32)
    rem_np[[20, 30]] = 1
    rem_np[[40]] = 0
    rem = torch.from_numpy(rem_np).cuda()
    tokens, status, rem_after, err = _run(x, eos, rem)
    t2, s2, r2, limit = sel.select_tokens(x.float().cpu().numpy(), eos.cpu().numpy(), rem_np)
    assert np.array_equal(tokens, x.argmax(dim=-1).cpu().numpy())
    assert np.array_equal(tokens, t2) and np.array_equal(status, s2) and np.array_equal(rem_after, r2)
    assert status[10] == sel.DONE | sel.EOS and status[20] == sel.DONE and status[40] == sel.DONE | sel.LIMIT
    assert err == 64 and limit


def test_reference_facing_step():
    """select_next_tokens + read_selection: the tokens the reference's
    argmax(keepdim=True) gives, the finish flags its loop computes, and its
    RuntimeError when a row had no tokens left."""
    from pagedserve_b200 import read_selection, select_next_tokens
    from pagedserve_b200.sampling import eos_tensor, remaining_tensor
    g = torch.Generator(device="cuda").manual_seed(5)
    logits = torch.randn(6, 2, 3000, generator=g, device="cuda").to(torch.bfloat16)
    logits[:, -1, [17, 99]] = -50.0   # only row 2 picks an EOS id
    logits[2, -1, 17] = 50.0
    eos = eos_tensor([17, 99], "cuda")
    rem = remaining_tensor([5, 5, 5, 3, 8, 2], [0, 4, 1, 1, 0, 0], "cuda")
    tokens, status = select_next_tokens(logits, eos, rem)
    assert torch.equal(tokens, logits[:, -1, :].argmax(dim=-1, keepdim=True))
    ids, done = read_selection(tokens, status)
    assert ids == tokens.view(-1).tolist()
    assert done == [False, True, True, False, False, False]
    assert rem.tolist() == [4, 0, 3, 1, 7, 1]
    rem.copy_(torch.tensor([4, 2, 3, 0, 7, 1], dtype=torch.int32))
    before = rem.tolist()
    tokens, status = select_next_tokens(logits, eos, rem)
    with pytest.raises(RuntimeError, match="generation limit") as info:
        read_selection(tokens, status)
    # the rows before the failing one keep their tokens, as in the reference's loop
    assert info.value.row == 3
    assert info.value.tokens == tokens.view(-1).tolist()
    assert rem.tolist() == [b - (0 if i == 3 else 1) for i, b in enumerate(before)]


def test_graph_capture_replays():
    """The selection captured in a CUDA graph (static buffers) and replayed
    over new logits counts the requests down step by step."""
    from pagedserve_b200 import ops
    b, v = 32, 10000
    logits = torch.zeros(b, v, device="cuda", dtype=torch.bfloat16)
    eos = torch.tensor([v + 5], dtype=torch.int64, device="cuda")  # never picked: rows end on the count
    rem = torch.full((b,), 3, dtype=torch.int32, device="cuda")
    tokens = torch.empty(b, dtype=torch.int64, device="cuda")
    status = torch.empty(b, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ops.select_tokens(logits, eos, rem, tokens=tokens, status=status)
        torch.cuda.synchronize()
        rem.fill_(3)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            ops.select_tokens(logits, eos, rem, tokens=tokens, status=status)
    for step in range(3):
        logits.copy_(torch.randn(b, v, device="cuda").to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(tokens, logits.argmax(dim=-1))
        assert rem.tolist() == [2 - step] * b
        assert bool((status == sel.DONE).all()) == (step == 2)
    graph.reset()


def _stream_geometry(vocab: int, cluster: int, esz: int):
    """The streaming kernel's split of a row, restated: CTA r of a cluster
    owns elements [r * chunk, (r + 1) * chunk); inside it, warp w owns 16-byte
    vectors [w0, w1) of an equal split over 8 warps; a warp streams them in
    4 KB pieces of 256 vectors, lane l holding vectors l, l + 32, ... of a
    piece.  Yields (slice start, slice vectors, per-warp (w0, w1))."""
    n = 16 // esz
    chunk = -(-(-(-vocab // cluster)) // n) * n
    for r in range(cluster):
        lo = r * chunk
        cnt = max(0, min(vocab, lo + chunk) - lo)
        nvec = cnt // n
        per = -(-nvec // 8)
        warps = [(min(nvec, w * per), min(nvec, min(nvec, w * per) + per)) for w in range(8)]
        yield lo, cnt, warps


def _planted_rows(vocab: int, cluster: int, esz: int):
    """Pairs of equal maxima planted where the index search changes hands:
    lane 31's last element of a warp's first piece against lane 0's first
    element of its second piece (the later lane wins the piece order, the
    earlier index wins the tie), a warp's last vector against the next
    warp's first, either side of a CTA slice boundary, and the ragged tail
    past the last whole vector."""
    n = 16 // esz
    pairs = []
    for lo, cnt, warps in _stream_geometry(vocab, cluster, esz):
        for w, (w0, w1) in enumerate(warps):
            if w1 - w0 > 256:  # the warp has a second piece
                a = lo + (w0 + 255) * n + n - 1   # lane 31, vector 7 of piece 0, last element
                b = lo + (w0 + 256) * n           # lane 0, vector 0 of piece 1, first element
                pairs.append((a, b))
                pairs.append((lo + (w0 + 255) * n, b))
                pairs.append((lo + (w0 + 31) * n + 3, lo + (w0 + 256 + 1) * n))  # lane 31 piece 0 vs lane 1 piece 1
            if w + 1 < 8 and warps[w + 1][1] > warps[w + 1][0] and w1 > w0:
                pairs.append((lo + w1 * n - 1, lo + w1 * n))
        if lo > 0 and cnt > 0:
            pairs.append((lo - 1, lo))
        tail = lo + (cnt // n) * n
        if tail < lo + cnt:  # elements past the slice's last whole vector
            pairs.append((tail - 1, lo + cnt - 1))
            pairs.append((lo + cnt - 1, lo + cnt - 1))
    pairs.append((vocab - 2, vocab - 1))
    return [p for p in pairs if 0 <= p[0] <= p[1] < vocab]


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
@pytest.mark.parametrize("vocab", [VOCAB, 70001])
@pytest.mark.parametrize("ctas", [1, 2, 8])
def test_first_maximum_at_stream_boundaries(dtype, vocab, ctas):
    """Row maxima tied across the pieces, warps and CTAs of the streaming
    kernel's schedule: the first index must win, as torch.argmax picks it."""
    from pagedserve_b200 import ops
    esz = 4 if dtype == "float32" else 2
    pairs = _planted_rows(vocab, ctas, esz)
    assert len(pairs) >= 4
    g = torch.Generator(device="cuda").manual_seed(vocab + ctas)
    # rows padded to a 16-byte pitch, so a ragged vocabulary still takes the
    # streaming kernel (its rows start on 16-byte boundaries)
    pitch = -(-vocab // 8) * 8
    x = torch.rand(len(pairs), pitch, generator=g, device="cuda").to(TORCH_DTYPES[dtype])[:, :vocab]
    for row, (a, b) in enumerate(pairs):
        x[row, a] = 8.0
        x[row, b] = 8.0
    eos = torch.tensor([vocab + 1], dtype=torch.int64, device="cuda")
    rem = torch.full((len(pairs),), 5, dtype=torch.int32, device="cuda")
    tokens, _, _, err = _run(x, eos, rem, ctas)
    assert err == 0
    want = np.array([a for a, _ in pairs])
    assert np.array_equal(tokens, want)
    assert np.array_equal(tokens, x.argmax(dim=-1).cpu().numpy())
