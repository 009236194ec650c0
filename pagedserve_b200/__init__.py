"""pagedserve_b200: PagedServe's paged-attention hot path for NVIDIA B200 (sm_100a).

Public surface:

* ``paged_decode_attention`` - drop-in for ``triton_paged_decode_attention``
  (pagedserve/attention/triton_paged_decode.py:98)
* ``write_tokens`` - batched replacement of the per-row ``write_token`` loop
* ``paged_decode_attention_with_write`` - both in one launch
* ``rope_and_write_tokens`` - the glue's rotary embedding fused with the write
* ``ops.reshape_and_cache / paged_decode / varlen_prefill / pack_step`` -
  tensor-level API over the C ABI (include/pagedserve_b200.h)
* ``select_next_tokens`` / ``read_selection`` - the step's greedy argmax and
  stop test on the device, one host sync per batch (replaces the per-row
  ``.item()`` loop of pagedserve/engine/continuous_batcher.py:333-360)
* ``PagedKVCache`` and friends - host-side block bookkeeping with the
  reference's interface
* ``SequenceDispatcher`` - places requests on the GPUs of a node (one
  process and one KV pool per GPU, no collective on the attention path)
"""

from . import ops
from .attention import (paged_decode_attention, paged_decode_attention_with_write, rope_and_write_tokens,
                        write_tokens)
from .paged_kv import BlockManager, BlockTable, KVCache, PagedKVCache
from .sampling import read_selection, select_next_tokens
from .sharding import SequenceDispatcher

__all__ = ["ops", "paged_decode_attention", "paged_decode_attention_with_write", "rope_and_write_tokens",
           "write_tokens", "select_next_tokens", "read_selection", "BlockManager", "BlockTable", "KVCache", "PagedKVCache", "SequenceDispatcher"]
__version__ = "0.1.0"
