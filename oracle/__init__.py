"""CPU oracle for the paged KV-cache hot path.  TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what the reference (prakhar-iit/mini-llm-inference-server,
`src/minillm/attention/` and `src/minillm/cache/`) computes on its hot path.  It exists to CHECK the
CUDA path and to time the reference's CPU algorithm beside it:

- only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
  `bench.py` may import it;
- the product package never imports it, and the product path fails loudly when its CUDA library is
  missing instead of falling back to anything here.

Parity pin: every function is checked against golden vectors that `tests/golden/make_golden.py`
produced by importing and running the reference itself (see `tests/test_oracle_golden.py`).
"""

from .paged_ref import (  # noqa: F401
    OracleMeta,
    build_metadata,
    compact_plan,
    copy_blocks,
    forward,
    gather,
    paged_attention,
    write_kv,
)
from .prefix_ref import block_hash, extend_chain, root_hash  # noqa: F401
