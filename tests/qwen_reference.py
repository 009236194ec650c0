"""The reference's decode and prefill forwards, with the oracle as attention.

``reference_decode`` follows PagedServe's ``_forward_paged_batch``
(pagedserve/model/engine.py:526-599) with ``batched_qwen_paged_attention``
(pagedserve/attention/batched_paged_attention.py:85-156) per layer: the
transformers Qwen2 modules for the embedding, norms, projections, rotary
embedding (``apply_rotary_pos_emb``), MLP and ``lm_head``; each row's rotated
key and value written at its position (``write_token``,
paged_kv_cache.py:187-200); attention by the float64 oracle
(``oracle.paged_attention.decode_attention``, the restatement of the
reference's ``vectorized_paged_attention``) over the pools.

Test infrastructure only: the library never imports this.
"""

from __future__ import annotations

import numpy as np
import torch
from transformers import Qwen2Config, Qwen2ForCausalLM
from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

from oracle import paged_attention as ora


def small_qwen(layers: int = 2, vocab: int = 512, dtype=torch.float32, device="cuda", seed: int = 0):
    """A random-init Qwen2 with Qwen2.5-0.5B's layer geometry (hidden 896,
    14q/2kv heads, d 64, SwiGLU 4864, RMSNorm eps 1e-6, rope theta 1e6,
    tied embeddings), ``layers`` layers and a small vocabulary; projection
    biases drawn too (the initialiser leaves them zero)."""
    cfg = Qwen2Config(hidden_size=896, intermediate_size=4864, num_hidden_layers=layers, num_attention_heads=14,
                      num_key_value_heads=2, vocab_size=vocab, max_position_embeddings=32768, rms_norm_eps=1e-6,
                      tie_word_embeddings=True, rope_theta=1e6, attn_implementation="eager")
    torch.manual_seed(seed)
    model = Qwen2ForCausalLM(cfg).eval()
    with torch.no_grad():
        for layer in model.model.layers:
            for proj in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj):
                proj.bias.normal_(0.0, 0.02)
            for norm in (layer.input_layernorm, layer.post_attention_layernorm):
                norm.weight.uniform_(0.5, 1.5)
        model.model.norm.weight.uniform_(0.5, 1.5)
    # the rotary inverse frequencies stay fp32, as in a model loaded with
    # from_pretrained(dtype=...) (engine.py:49-53); a blanket .to(dtype) would
    # round them
    inv_freq = model.model.rotary_emb.inv_freq.clone()
    model = model.to(device=device, dtype=dtype)
    model.model.rotary_emb.inv_freq = inv_freq.to(device)
    return model


@torch.no_grad()
def reference_decode(model, input_ids: torch.Tensor, positions, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     tables, block_size: int = 16) -> torch.Tensor:
    """Logits ``[B, V]`` of one decode token per row; writes each row's K/V
    into ``k_cache / v_cache`` (torch tensors) as the reference does."""
    m = model.model
    bsz = input_ids.shape[0]
    dev = input_ids.device
    cfg = model.config
    hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    d = cfg.hidden_size // hq
    position_ids = torch.tensor(positions, dtype=torch.long, device=dev).view(bsz, 1)
    hidden = m.embed_tokens(input_ids.view(bsz, 1))
    cos, sin = m.rotary_emb(hidden, position_ids)
    lens = [p + 1 for p in positions]
    for li, layer in enumerate(m.layers):
        residual = hidden
        x = layer.input_layernorm(hidden)
        a = layer.self_attn
        q = a.q_proj(x).view(bsz, 1, -1, d).transpose(1, 2)
        k = a.k_proj(x).view(bsz, 1, -1, d).transpose(1, 2)
        v = a.v_proj(x).view(bsz, 1, -1, d).transpose(1, 2)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        for row, pos in enumerate(positions):
            blk, off = tables[row][pos // block_size], pos % block_size
            k_cache[li, blk, :, off, :] = k[row, :, 0, :]
            v_cache[li, blk, :, off, :] = v[row, :, 0, :]
        kc = k_cache.float().cpu().numpy()
        vc = v_cache.float().cpu().numpy()
        attn = ora.decode_attention(q[:, :, 0, :].float().cpu().numpy(), kc, vc, tables, lens, li)
        attn = torch.from_numpy(attn).to(device=dev, dtype=hidden.dtype)       # [B, Hq, D]
        out = a.o_proj(attn.reshape(bsz, 1, hq * d))
        hidden = residual + out
        residual = hidden
        hidden = residual + layer.mlp(layer.post_attention_layernorm(hidden))
    return model.lm_head(m.norm(hidden))[:, 0, :]


@torch.no_grad()
def reference_prefill_logits(model, prompt: torch.Tensor) -> torch.Tensor:
    """Last-position logits of one prompt through the full transformers
    forward (eager causal attention) - what ``_forward_paged`` computes for a
    prompt with ``paged_attention`` as its attention (engine.py:601-650)."""
    return model(prompt.view(1, -1)).logits[0, -1]


@torch.no_grad()
def reference_greedy(model, prompt: torch.Tensor, max_new_tokens: int) -> list[int]:
    """Greedy continuation by full recomputation: the token sequence any
    correct paged engine must reproduce (fp32, no ties)."""
    ids = prompt.view(1, -1)
    out = []
    for _ in range(max_new_tokens):
        nxt = int(model(ids).logits[0, -1].argmax())
        out.append(nxt)
        ids = torch.cat([ids, torch.tensor([[nxt]], device=ids.device)], dim=1)
    return out


def random_tables(rng: np.random.Generator, lens, num_blocks: int, block_size: int = 16):
    """Fragmented block tables: each request's blocks a slice of one random permutation of the pool."""
    perm = rng.permutation(num_blocks)
    tables, at = [], 0
    for n in lens:
        k = -(-int(n) // block_size)
        tables.append([int(b) for b in perm[at:at + k]])
        at += k
    return tables
