"""Generate the golden vectors by running the REFERENCE itself (prakhar-iit/mini-llm-inference-server).

Run in a container where the reference is mounted (it is Python: nothing is compiled):

    MINILLM_REF_SRC=/path/to/mini-llm-inference-server/src python tests/golden/make_golden.py

It imports the reference's own `write_kv`, `TorchRefBackend.forward` (write + paged attention),
`AttentionMetadata.build` and prefix-cache hash chain, runs them on the seeded inputs of `cases.py`
(CPU, fp32) and writes:
- attention.npz   per case: SHA-256 of the inputs and the reference's [N, H, Dh] output
- append_cast.npz fp32 rows written into bf16 and fp16 pools by the reference: the stored bit patterns
- metadata.json   AttentionMetadata fields for a set of ragged steps (incl. tests/test_paged.py:41-50)
- prefix.json     root and block hashes (incl. tests/test_prefix_cache.py:33-40)
- interface.json  the field names of the reference's AttentionMetadata dataclass and the abstract methods of
                  its AttentionBackend: the object shape an unmodified reference engine hands a backend
Nothing here runs on the GPU box; the tests only read the files it wrote.
"""

from __future__ import annotations

import dataclasses
import inspect
import json
import os
import random
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
if "MINILLM_REF_SRC" not in os.environ:
    sys.exit("set MINILLM_REF_SRC to the reference's src/ directory (see the docstring)")
sys.path.insert(0, os.environ["MINILLM_REF_SRC"])

import cases  # noqa: E402
from minillm.attention.base import AttentionBackend  # noqa: E402
from minillm.attention.metadata import AttentionMetadata, SeqStep  # noqa: E402
from minillm.attention.paged_torch_ref import write_kv  # noqa: E402
from minillm.attention.torch_ref import TorchRefBackend  # noqa: E402
from minillm.cache.prefix import block_hash, extend_chain, root_hash  # noqa: E402


def reference_forward(case: cases.PagedCase) -> torch.Tensor:
    meta = AttentionMetadata.build([SeqStep(c, n, list(b)) for c, n, b in case.seqs], case.bs, "cpu")
    k_pool, v_pool = case.k_pool.clone(), case.v_pool.clone()
    with torch.inference_mode():
        out = TorchRefBackend().forward(case.q, case.k, case.v, k_pool, v_pool, meta)
    # the write must land exactly where slot_mapping says (paged_torch_ref.py:27-28)
    flat = k_pool.view(-1, case.hkv, case.dh)
    assert torch.equal(flat[meta.slot_mapping], case.k)
    return out


def attention_golden() -> dict:
    out = {}
    for case in cases.attention_cases():
        out[f"{case.name}.digest"] = np.array(case.digest())
        out[f"{case.name}.out"] = reference_forward(case).numpy()
        print(f"  {case.name}: N={case.q.shape[0]} H={case.h} Hkv={case.hkv} Dh={case.dh}")
    return out


def append_golden() -> dict:
    x = cases.cast_rows()
    n, hkv, dh = x.shape
    out = {"rows.digest": np.array(__import__("hashlib").sha256(x.numpy().tobytes()).hexdigest())}
    slots = torch.tensor(random.Random(0).sample(range(8 * cases.BS), n))
    for name, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        k_pool = torch.zeros(8, cases.BS, hkv, dh, dtype=dt)
        v_pool = torch.zeros_like(k_pool)
        write_kv(k_pool, v_pool, slots, x, -x)
        k_rows = k_pool.view(-1, hkv, dh)[slots].view(torch.int16).numpy().view(np.uint16)
        v_rows = v_pool.view(-1, hkv, dh)[slots].view(torch.int16).numpy().view(np.uint16)
        out[f"{name}.k_bits"] = k_rows
        out[f"{name}.v_bits"] = v_rows
    out["slots"] = slots.numpy()
    return out


def metadata_golden() -> list:
    rng = random.Random(9)
    steps_list = [
        (4, [(3, 1, [7]), (0, 5, [2, 9])]),  # tests/test_paged.py:41-50
        (16, [(c, n, b) for (c, n), b in zip(cases.MIXED_STEPS, [[1, 2, 3], [4, 5, 6, 7, 8, 9],
                                                                 [10, 11, 12, 13, 14], [15], [16 + i for i in range(19)]])]),
    ]
    for _ in range(4):
        seqs = []
        for _ in range(rng.randint(1, 9)):
            cached, new = rng.randint(0, 100), rng.randint(1, 40)
            need = -(-(cached + new) // 16) + rng.randint(0, 2)  # tables may hold spare blocks
            seqs.append((cached, new, [rng.randrange(500) for _ in range(need)]))
        steps_list.append((16, seqs))
    out = []
    for bs, seqs in steps_list:
        meta = AttentionMetadata.build([SeqStep(c, n, list(b)) for c, n, b in seqs], bs, "cpu")
        out.append({
            "block_size": bs, "seqs": [[c, n, list(b)] for c, n, b in seqs],
            "query_start_loc": meta.query_start_loc, "seq_lens": meta.seq_lens,
            "positions": meta.positions.tolist(), "slot_mapping": meta.slot_mapping.tolist(),
            "block_tables": meta.block_tables.tolist(), "logits_index": meta.logits_index.tolist(),
            "kv_indptr": meta.kv_indptr.tolist(), "kv_indices": meta.kv_indices.tolist(),
            "kv_last_page_len": meta.kv_last_page_len.tolist(),
        })
    try:
        AttentionMetadata.build([SeqStep(0, 5, [2])], 4, "cpu")
    except ValueError as e:
        out.append({"error": str(e), "block_size": 4, "seqs": [[0, 5, [2]]]})
    return out


def prefix_golden() -> dict:
    keys = [
        {"model": "m@abc", "kv_dtype": "bfloat16", "layout": "NHD", "block_size": 16, "salt": ""},  # test :35
        {"salt": ""}, {"salt": "t"}, {"model": "llama-3.1-8b@r1", "salt": "tenant-ä"},
    ]
    roots = [root_hash(k).hex() for k in keys]
    r = random.Random(4)
    chains = []
    for i, k in enumerate(keys):
        toks = [r.randrange(128256) for _ in range(16 * 5 + 3)]
        chain: list[bytes] = []
        extend_chain(chain, root_hash(k), toks, 5, 16)
        chains.append({"key": i, "tokens": toks, "chain": [c.hex() for c in chain]})
    single = block_hash(root_hash(keys[0]), list(range(100, 116))).hex()
    return {"keys": keys, "roots": roots, "chains": chains, "block_100_115": single}


def interface_golden() -> dict:
    return {"metadata_fields": [f.name for f in dataclasses.fields(AttentionMetadata)],
            "backend_abstract_methods": sorted(AttentionBackend.__abstractmethods__),
            "forward_parameters": list(inspect.signature(AttentionBackend.forward).parameters)}


def main() -> None:
    torch.manual_seed(0)
    print("attention (reference TorchRefBackend.forward, fp32 CPU):")
    np.savez_compressed(HERE / "attention.npz", **attention_golden())
    np.savez_compressed(HERE / "append_cast.npz", **append_golden())
    (HERE / "metadata.json").write_text(json.dumps(metadata_golden()) + "\n")
    (HERE / "prefix.json").write_text(json.dumps(prefix_golden(), ensure_ascii=False) + "\n")
    (HERE / "interface.json").write_text(json.dumps(interface_golden()) + "\n")
    for f in sorted(HERE.glob("*.npz")) + sorted(HERE.glob("*.json")):
        print(f"  wrote {f.name}: {f.stat().st_size} bytes")


if __name__ == "__main__":
    main()
