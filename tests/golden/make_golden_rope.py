"""Golden vectors for the fused RoPE + KV write, from the reference's own code.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden_rope.py --reference <PagedServe checkout>

The reference rotates q and k in its decode glue with ``apply_rotary_pos_emb``
as imported by pagedserve/attention/batched_paged_attention.py:8 (the
transformers Qwen2 function) on the ``(cos, sin)`` position embeddings its
engine computes once per step with the model's rotary embedding
(pagedserve/model/engine.py:572-575).  This script builds that rotary
embedding for Qwen2.5-0.5B's geometry (head_dim 64, rope theta 1e6), computes
cos/sin for seeded positions, applies the reference's ``apply_rotary_pos_emb``
to seeded q/k on the CPU, and stores inputs and outputs in
``tests/golden/rope_outputs.npz``.  Nothing on the GPU box reads the
reference: the tests only read that file.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

# (name, dtype, tokens, positions drawn below this bound)
CASES = [("decode_bf16", "bfloat16", 8, 32768), ("prefill_bf16", "bfloat16", 24, 2048),
         ("prefill_f16", "float16", 16, 4096), ("prefill_f32", "float32", 16, 32768)]
HQ, HKV, D, THETA = 14, 2, 64, 1e6


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of a PagedServe checkout (the directory holding the pagedserve package)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)

    import torch
    from pagedserve.attention.batched_paged_attention import apply_rotary_pos_emb
    from transformers.models.qwen2.configuration_qwen2 import Qwen2Config
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding

    config = Qwen2Config(hidden_size=HQ * D, num_attention_heads=HQ, num_key_value_heads=HKV,
                         max_position_embeddings=32768, rope_parameters={"rope_type": "default", "rope_theta": THETA})
    rotary = Qwen2RotaryEmbedding(config)
    dtypes = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
    arrays: dict[str, np.ndarray] = {}
    for i, (name, dtype, tokens, bound) in enumerate(CASES):
        dt = dtypes[dtype]
        g = torch.Generator().manual_seed(100 + i)
        positions = torch.randint(0, bound, (tokens,), generator=g)
        positions[0] = 0
        q = torch.randn(tokens, HQ, D, generator=g).to(dt)
        k = torch.randn(tokens, HKV, D, generator=g).to(dt)
        # the engine's call: one row of position ids, embeddings for every token
        cos, sin = rotary(q, positions.view(1, tokens))
        # the glue's layout: [B, H, S, D] with cos/sin [B, S, D]
        q_embed, k_embed = apply_rotary_pos_emb(q.transpose(0, 1).unsqueeze(0), k.transpose(0, 1).unsqueeze(0),
                                                cos, sin)
        arrays[f"{name}/positions"] = positions.numpy().astype(np.int64)
        arrays[f"{name}/q"] = q.float().numpy()
        arrays[f"{name}/k"] = k.float().numpy()
        arrays[f"{name}/cos"] = cos[0].float().numpy()
        arrays[f"{name}/sin"] = sin[0].float().numpy()
        arrays[f"{name}/q_embed"] = q_embed[0].transpose(0, 1).float().numpy()
        arrays[f"{name}/k_embed"] = k_embed[0].transpose(0, 1).float().numpy()
    np.savez_compressed(os.path.join(HERE, "rope_outputs.npz"), **arrays)
    print(f"wrote {len(arrays)} arrays")


if __name__ == "__main__":
    main()
