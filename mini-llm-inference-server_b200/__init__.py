"""B200-native (sm_100a) paged KV-cache hot path of prakhar-iit/mini-llm-inference-server.

Drop-in beside the reference's backends: `get_backend("b200")` returns an `AttentionBackend` whose
`forward(q, k, v, k_cache, v_cache, meta)` appends the step's k/v through `slot_mapping` and runs paged
attention over `block_tables` on hand-written CUDA kernels (C ABI: include/mlb_paged_kv.h, library
`_mlb_paged_kv.so` built in-tree by `build.py`).  The cache side keeps the reference's `PagedKVCache`,
`PrefixCache` and `BlockManager` API and adds block copy-on-write and compaction.

The directory name is not a Python identifier; import it with
`importlib.import_module("mini-llm-inference-server_b200")`.
"""

from . import ops
from .attention import AttentionBackend, AttentionMetadata, B200Backend, DeviceFault, SeqStep, get_backend
from .cache import BLOCK_SIZE, BlockManager, KVShape, PagedKVCache, PagedStep, PrefixCache
from .ops import AttentionPlan, Workspace, block_copy, kv_append, paged_attention, plan_attention

__all__ = ["AttentionBackend", "AttentionMetadata", "AttentionPlan", "B200Backend", "BLOCK_SIZE", "BlockManager",
           "DeviceFault",
           "KVShape", "PagedKVCache", "PagedStep", "PrefixCache", "SeqStep", "Workspace", "block_copy",
           "get_backend", "kv_append", "ops", "paged_attention", "plan_attention"]
