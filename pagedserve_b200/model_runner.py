"""Qwen2 forward passes over the paged KV pool, on this package's kernels.

The reference's model runner executes Qwen2.5 through transformers' modules
and swaps in its own attention per layer:

* ``_forward_paged_batch`` (pagedserve/model/engine.py:526-599): one decode
  token per request, ``batched_qwen_paged_attention`` per layer
  (pagedserve/attention/batched_paged_attention.py:15-156: q/k/v
  projections, ``apply_rotary_pos_emb``, a ``write_token`` per row, paged
  decode attention, ``o_proj``);
* ``_forward_paged`` (engine.py:601-650): the prefill of ONE request,
  ``qwen_paged_attention`` per layer (qwen_paged_attention.py:12-135).

``PagedModelRunner`` runs the same layer structure for a whole batch:

* decode: RoPE + the KV write of every row in one launch
  (``rope_reshape_and_cache``), split-K paged decode, and the residual /
  RMSNorm / SiLU glue as one launch each (``add_rms_norm``,
  ``silu_and_mul``); the projections, ``o_proj``, the MLP matrices and the
  tied ``lm_head`` are cuBLAS GEMMs through ``torch.nn.functional.linear``
  (q/k/v fused into one GEMM, gate/up into another);
* prefill: every admitted prompt in ONE packed pass (``cu_seqlens``), with
  ``varlen_prefill`` as the attention, instead of one request at a time; only
  each sequence's last row reaches the final norm and ``lm_head``.

Every launch is asynchronous on the current stream and the passes allocate
only through PyTorch's caching allocator, so both can be captured in CUDA
graphs (``DecodeGraph`` and ``PrefillGraph`` in ``serving.py``).
"""

from __future__ import annotations

import dataclasses
import math

import torch
import torch.nn.functional as F

from . import ops


@dataclasses.dataclass(frozen=True)
class QwenConfig:
    """The Qwen2 geometry the runner needs (defaults: Qwen2.5-0.5B)."""

    hidden: int = 896
    layers: int = 24
    q_heads: int = 14
    kv_heads: int = 2
    head_dim: int = 64
    intermediate: int = 4864
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    max_positions: int = 32768

    @classmethod
    def from_hf(cls, cfg) -> "QwenConfig":
        """From a transformers ``Qwen2Config``."""
        return cls(hidden=cfg.hidden_size, layers=cfg.num_hidden_layers, q_heads=cfg.num_attention_heads,
                   kv_heads=cfg.num_key_value_heads, head_dim=cfg.hidden_size // cfg.num_attention_heads,
                   intermediate=cfg.intermediate_size, vocab=cfg.vocab_size, rms_eps=cfg.rms_norm_eps,
                   rope_theta=float(getattr(cfg, "rope_theta", None) or cfg.rope_parameters["rope_theta"]),
                   max_positions=cfg.max_position_embeddings)

    @property
    def qkv_width(self) -> int:
        return (self.q_heads + 2 * self.kv_heads) * self.head_dim

    def weight_bytes(self, esz: int = 2) -> int:
        """Bytes of weights one decode step streams (the tied embedding once, as lm_head)."""
        per_layer = (self.qkv_width * self.hidden + self.qkv_width + self.hidden * self.q_heads * self.head_dim
                     + 2 * self.intermediate * self.hidden + self.hidden * self.intermediate + 2 * self.hidden)
        return esz * (self.layers * per_layer + self.vocab * self.hidden + self.hidden)


class QwenWeights:
    """Weights in the layout the runner launches on: per layer the fused
    q|k|v projection ``[(Hq + 2 Hkv) D, H]`` with its bias, ``o_proj``
    ``[H, Hq D]``, the fused gate|up projection ``[2 I, H]``, ``down_proj``
    ``[H, I]`` and the two RMSNorm weights; the embedding (tied to
    ``lm_head``) and the final norm."""

    def __init__(self, cfg: QwenConfig, embed, norm, ln1, ln2, qkv, qkv_bias, o, gate_up, down, lm_head=None):
        self.cfg = cfg
        self.embed, self.norm = embed, norm
        self.ln1, self.ln2 = ln1, ln2
        self.qkv, self.qkv_bias, self.o = qkv, qkv_bias, o
        self.gate_up, self.down = gate_up, down
        self.lm_head = embed if lm_head is None else lm_head

    @property
    def dtype(self) -> torch.dtype:
        return self.embed.dtype

    @property
    def device(self) -> torch.device:
        return self.embed.device

    @classmethod
    def random(cls, cfg: QwenConfig, device, dtype=torch.bfloat16, seed: int = 0, std: float = 0.02
               ) -> "QwenWeights":
        """Random-init weights: N(0, std) matrices, embedding and biases
        (transformers' Qwen2 initialiser draws matrices and the embedding
        from N(0, 0.02)), norms at one, lm_head tied to the embedding."""
        g = torch.Generator(device=device)
        g.manual_seed(seed)

        def mat(*shape):
            return torch.empty(shape, device=device, dtype=dtype).normal_(0.0, std, generator=g)

        h, d = cfg.hidden, cfg.head_dim
        ones = lambda n: torch.ones(n, device=device, dtype=dtype)
        L = cfg.layers
        return cls(cfg, embed=mat(cfg.vocab, h), norm=ones(h), ln1=[ones(h) for _ in range(L)],
                   ln2=[ones(h) for _ in range(L)], qkv=[mat(cfg.qkv_width, h) for _ in range(L)],
                   qkv_bias=[mat(cfg.qkv_width) for _ in range(L)], o=[mat(h, cfg.q_heads * d) for _ in range(L)],
                   gate_up=[mat(2 * cfg.intermediate, h) for _ in range(L)],
                   down=[mat(h, cfg.intermediate) for _ in range(L)])

    @classmethod
    def from_hf(cls, model) -> "QwenWeights":
        """From a transformers ``Qwen2ForCausalLM`` (the module the reference
        engine loads, engine.py:49-53); tensors are copied into the fused layout."""
        cfg = QwenConfig.from_hf(model.config)
        m = model.model
        ln1, ln2, qkv, qkv_b, o, gu, down = [], [], [], [], [], [], []
        for layer in m.layers:
            a, mlp = layer.self_attn, layer.mlp
            ln1.append(layer.input_layernorm.weight.detach().clone())
            ln2.append(layer.post_attention_layernorm.weight.detach().clone())
            qkv.append(torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight]).detach().contiguous())
            qkv_b.append(torch.cat([a.q_proj.bias, a.k_proj.bias, a.v_proj.bias]).detach().contiguous())
            o.append(a.o_proj.weight.detach().clone())
            gu.append(torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight]).detach().contiguous())
            down.append(mlp.down_proj.weight.detach().clone())
        embed = m.embed_tokens.weight.detach().clone()
        head = model.lm_head.weight.detach()
        tied = head.data_ptr() == m.embed_tokens.weight.data_ptr()
        return cls(cfg, embed=embed, norm=m.norm.weight.detach().clone(), ln1=ln1, ln2=ln2, qkv=qkv, qkv_bias=qkv_b,
                   o=o, gate_up=gu, down=down, lm_head=None if tied else head.clone())


def rope_tables(cfg: QwenConfig, device, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin rows ``[max_positions, D]`` of Qwen2's default rotary
    embedding, evaluated as transformers does for ``position_ids``
    (fp32 angles position x inv_freq, duplicated halves, cos/sin in fp32,
    then cast to the model dtype), so gathering row p gives the engine's
    ``position_embeddings`` for position p (engine.py:572-575)."""
    d = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64, device=device).float() / d))
    pos = torch.arange(cfg.max_positions, device=device, dtype=torch.float32)
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


class PagedModelRunner:
    """Batched Qwen2 decode and packed prefill over a ``PagedKVCache``'s pools."""

    def __init__(self, weights: QwenWeights, k_cache: torch.Tensor, v_cache: torch.Tensor, block_size: int = 16):
        cfg = weights.cfg
        if k_cache.shape[0] != cfg.layers or tuple(k_cache.shape[2:]) != (cfg.kv_heads, block_size, cfg.head_dim):
            raise ValueError("the pools do not match the model: expected "
                             f"[{cfg.layers}, blocks, {cfg.kv_heads}, {block_size}, {cfg.head_dim}]")
        if k_cache.dtype != weights.dtype:
            raise ValueError("pool and weight dtypes differ")
        self.cfg, self.w = cfg, weights
        self.k_cache, self.v_cache = k_cache, v_cache
        self.block_size = block_size
        self.cos, self.sin = rope_tables(cfg, weights.device, weights.dtype)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)

    # -- pieces shared by both passes -----------------------------------------
    def _qkv(self, x: torch.Tensor, layer: int):
        cfg = self.cfg
        t, hq, hkv, d = x.shape[0], cfg.q_heads, cfg.kv_heads, cfg.head_dim
        qkv = F.linear(x, self.w.qkv[layer], self.w.qkv_bias[layer])
        q = qkv[:, : hq * d].view(t, hq, d)
        k = qkv[:, hq * d:(hq + hkv) * d].view(t, hkv, d)
        v = qkv[:, (hq + hkv) * d:].view(t, hkv, d)
        return q, k, v

    def _mlp(self, x: torch.Tensor, layer: int) -> torch.Tensor:
        return F.linear(ops.silu_and_mul(F.linear(x, self.w.gate_up[layer])), self.w.down[layer])

    def _layers(self, tokens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor, attend, want_keys: bool,
                last_rows=None) -> torch.Tensor:
        """Embedding, the decoder layers and the final norm + lm_head.

        ``attend(q_rot, k_rot, v, layer)`` is the attention of one layer over
        rotated queries (the rotated keys and the values are already in the
        pool; ``k_rot`` is None unless ``want_keys``); ``last_rows`` picks
        the rows that reach ``lm_head``."""
        cfg, w = self.cfg, self.w
        eps = cfg.rms_eps
        residual = F.embedding(tokens, w.embed)
        cos = self.cos.index_select(0, positions)
        sin = self.sin.index_select(0, positions)
        x = ops.add_rms_norm(residual, w.ln1[0], eps)
        mlp_out = None
        for layer in range(cfg.layers):
            if layer > 0:
                ops.add_rms_norm(mlp_out, w.ln1[layer], eps, residual=residual, out=x)
            q, k, v = self._qkv(x, layer)
            q_rot, k_rot = ops.rope_reshape_and_cache(q, k, v, cos, sin, self.k_cache, self.v_cache, slots, layer,
                                                      key_out=None if want_keys else False)
            attn = attend(q_rot, k_rot, v, layer)
            o = F.linear(attn.view(attn.shape[0], -1), w.o[layer])
            ops.add_rms_norm(o, w.ln2[layer], eps, residual=residual, out=x)
            mlp_out = self._mlp(x, layer)
        if last_rows is not None:
            mlp_out = mlp_out.index_select(0, last_rows)
            residual = residual.index_select(0, last_rows)
        h = ops.add_rms_norm(mlp_out, w.norm, eps, residual=residual)
        return F.linear(h, w.lm_head)

    # -- decode ---------------------------------------------------------------
    def decode(self, tokens: torch.Tensor, positions: torch.Tensor, block_tables: torch.Tensor,
               context_lens: torch.Tensor, slots: torch.Tensor, max_context: int | None = None) -> torch.Tensor:
        """One decode token per row: ``tokens, positions, slots [B]`` int64
        (token b sits at ``positions[b]`` and its K/V goes to ``slots[b]``),
        ``block_tables [B, W]`` / ``context_lens [B]`` int32 with
        ``context_lens[b] == positions[b] + 1``.  Returns logits ``[B, V]``
        (``_forward_paged_batch``'s ``[B, 1, V]`` without the unit axis)."""
        max_context = block_tables.shape[1] * self.block_size if max_context is None else max_context

        def attend(q_rot, _k, _v, layer):
            return ops.paged_decode(q_rot, self.k_cache, self.v_cache, block_tables, context_lens, layer,
                                    scale=self.scale, max_context=max_context)
        return self._layers(tokens, positions, slots, attend, want_keys=False)

    # -- packed prefill ----------------------------------------------------------
    def prefill(self, tokens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor, cu_seqlens: torch.Tensor,
                max_seqlen: int, last_rows: torch.Tensor) -> torch.Tensor:
        """Prompts packed back to back: ``tokens, positions, slots [T]``
        int64 (a negative slot is a padding token: its K/V is not stored),
        ``cu_seqlens [B+1]`` int32, each sequence causal within itself and
        starting at position 0.  Returns the logits of ``last_rows [B]``
        (each sequence's last token), ``[B, V]``."""
        def attend(q_rot, k_rot, v, layer):
            return ops.varlen_prefill(q_rot, k_rot, v, cu_seqlens, max_seqlen, scale=self.scale)
        return self._layers(tokens, positions, slots, attend, want_keys=True, last_rows=last_rows)

    # -- prefill and decode in one pass --------------------------------------------
    def mixed(self, tokens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor, prefill_tokens: int,
              prefill_cu: torch.Tensor, max_seqlen: int, block_tables: torch.Tensor, context_lens: torch.Tensor,
              last_rows: torch.Tensor, max_context: int | None = None) -> torch.Tensor:
        """One engine step's prompts and decode rows in ONE pass.

        Rows ``0 .. prefill_tokens - 1`` of ``tokens, positions, slots`` are
        prompts packed back to back (``prefill_cu [S+1]``, causal within each,
        starting at position 0), the remaining ``B`` rows one decode token per
        running request (``block_tables [B, W]``, ``context_lens [B]`` =
        position + 1).  Every row goes through the same embedding, norms,
        projections, RoPE + KV write and MLP launches; only the attention
        splits: ``varlen_prefill`` over the prompt rows, ``paged_decode`` over
        the decode rows.  Returns the logits of ``last_rows`` (each prompt's
        last row, then the decode rows).  Equal, row for row, to ``prefill``
        and ``decode`` run apart: rows never read each other outside the
        attention."""
        tp = int(prefill_tokens)
        max_context = block_tables.shape[1] * self.block_size if max_context is None else max_context

        def attend(q_rot, k_rot, v, layer):
            out = torch.empty_like(q_rot)
            if tp > 0:
                ops.varlen_prefill(q_rot[:tp], k_rot[:tp], v[:tp], prefill_cu, max_seqlen, scale=self.scale,
                                   out=out[:tp])
            if q_rot.shape[0] > tp:
                ops.paged_decode(q_rot[tp:], self.k_cache, self.v_cache, block_tables, context_lens, layer,
                                 scale=self.scale, out=out[tp:], max_context=max_context)
            return out
        return self._layers(tokens, positions, slots, attend, want_keys=True, last_rows=last_rows)

