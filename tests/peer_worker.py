"""One rank of the two-GPU check in test_peer_gpu.py (run under torchrun): KV-head-sharded forward with the
p2p output gather (flagged packets, and plain stores + barrier) equals the NCCL all-gather bit for bit, over
several forwards (both slots and both packet areas reused), from the full rows (`forward`) and from each
rank's own heads (`forward_local`), and matches the fp32 oracle within the bf16 tolerance."""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from importlib import import_module
from pathlib import Path

TESTS = Path(__file__).resolve().parent
sys.path[:0] = [str(TESTS.parent), str(TESTS / "golden"), str(TESTS)]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import cases  # noqa: E402
from paged_helpers import assert_close, device_case, oracle_forward  # noqa: E402


def main() -> None:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
    mlb = import_module("mini-llm-inference-server_b200")
    sharding = import_module("mini-llm-inference-server_b200.sharding")
    p2p = sharding.KVHeadShardedBackend(transport="p2p", exchange="packets")
    p2b = sharding.KVHeadShardedBackend(transport="p2p", exchange="barrier")
    nccl = sharding.KVHeadShardedBackend(transport="nccl")
    for case in (cases.mixed_step(4, 32, 8, 128), cases.llama_decode(21, 6, 512, 4096), cases.boundaries(6, 32, 8, 64)):
        dtype = torch.bfloat16
        t = device_case(case, dtype, dev)
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], case.bs, dev)
        ks = sharding.head_range(rank, world, case.hkv)
        pools = [t[name][:, :, ks].contiguous() for name in ("k_pool", "v_pool", "k_pool", "v_pool")]
        expected = oracle_forward(case, dtype)[0]
        qs = sharding.head_range(rank, world, case.h)
        for _ in range(3):  # slots 0, 1, 0 ...
            got = p2p.forward(t["q"], t["k"], t["v"], pools[0], pools[1], meta).clone()
            want = nccl.forward(t["q"], t["k"], t["v"], pools[2], pools[3], meta)
            assert torch.equal(got, want), f"rank {rank}: p2p gather differs from NCCL ({case.name})"
            assert_close(got, expected, dtype)
            got = p2b.forward(t["q"], t["k"], t["v"], pools[0], pools[1], meta)
            assert torch.equal(got, want), f"rank {rank}: p2p gather with barrier differs from NCCL ({case.name})"
            # the same step from this rank's own heads only (forward_local), both transports
            loc = p2p.forward_local(t["q"][:, qs].contiguous(), t["k"][:, ks].contiguous(),
                                    t["v"][:, ks].contiguous(), pools[0], pools[1], meta).clone()
            assert torch.equal(loc, want), f"rank {rank}: p2p forward_local differs ({case.name})"
            loc = nccl.forward_local(t["q"][:, qs], t["k"][:, ks], t["v"][:, ks], pools[2], pools[3], meta)
            assert torch.equal(loc, want), f"rank {rank}: NCCL forward_local differs ({case.name})"
    for b in (p2p, p2b):
        b.peers.raise_errors()
        b.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: peer gather ok", flush=True)


if __name__ == "__main__":
    main()
