"""KV-head sharding on CPU ranks (torch.distributed gloo, world size 2 and 4): each rank holds only its KV
heads' pools, attends with an oracle-backed inner backend, and the all-gathered output equals the
unsharded oracle, from the full rows (`forward`) and from each rank's own heads (`forward_local`).  Also: a
rank that dies before the collective makes the others fail fast (host-side
failure injection; no GPU involved)."""

from __future__ import annotations

import os
import socket
import sys
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import GOLDEN, PACKAGE, REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleInner:
    """A CPU stand-in for B200Backend inside the sharded wrapper (the test's checker, not the product)."""

    name = "oracle"

    def prefill(self, q, k, v, key_valid=None, **kwargs):
        raise NotImplementedError

    def forward(self, q, k, v, k_cache, v_cache, meta):
        import oracle

        return oracle.forward(q, k, v, k_cache, v_cache, meta)


def _worker(rank: int, world: int, port: int, mode: str, result_path: str) -> None:
    sys.path[:0] = [str(REPO), str(GOLDEN)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    from importlib import import_module

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        sharding = import_module(PACKAGE + ".sharding")
        import cases
        import oracle

        case = cases.mixed_step(4, 32, 8, 128)
        meta = oracle.build_metadata(case.seqs, case.bs)
        ks = sharding.head_range(rank, world, case.hkv)
        k_pool = case.k_pool[:, :, ks].contiguous()
        v_pool = case.v_pool[:, :, ks].contiguous()
        backend = sharding.KVHeadShardedBackend(inner=OracleInner())
        if mode == "die" and rank == world - 1:
            os._exit(3)  # this rank leaves before the collective, between steps
        out = backend.forward(case.q, case.k, case.v, k_pool, v_pool, meta)
        if rank == 0:
            torch.save(out, result_path)
        # the same step from this rank's own heads only (as a column-parallel QKV projection leaves them)
        qs = sharding.head_range(rank, world, case.h)
        k_pool_l = case.k_pool[:, :, ks].contiguous()
        v_pool_l = case.v_pool[:, :, ks].contiguous()
        out_l = backend.forward_local(case.q[:, qs], case.k[:, ks], case.v[:, ks], k_pool_l, v_pool_l, meta)
        assert torch.equal(out_l, out)
        # this rank's slice of the pools was written exactly like the unsharded write
        full_k = case.k_pool.clone()
        oracle.write_kv(full_k, case.v_pool.clone(), meta.slot_mapping, case.k, case.v)
        assert torch.equal(k_pool, full_k[:, :, ks])
        dist.destroy_process_group()
    except Exception:
        with open(result_path + f".err{rank}", "w") as f:
            f.write(traceback.format_exc())
        raise


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_output_equals_unsharded_oracle(tmp_path, world):
    import cases
    import oracle

    path = str(tmp_path / "out.pt")
    mp.start_processes(_worker, args=(world, _free_port(), "ok", path), nprocs=world, start_method="spawn")
    case = cases.mixed_step(4, 32, 8, 128)
    meta = oracle.build_metadata(case.seqs, case.bs)
    expected = oracle.forward(case.q, case.k, case.v, case.k_pool.clone(), case.v_pool.clone(), meta)
    torch.testing.assert_close(torch.load(path), expected, atol=1e-6, rtol=1e-6)


def test_a_rank_that_dies_fails_the_others_fast(tmp_path):
    path = str(tmp_path / "out.pt")
    with pytest.raises(mp.ProcessExitedException):
        mp.start_processes(_worker, args=(2, _free_port(), "die", path), nprocs=2, start_method="spawn")
    assert not os.path.exists(path)


def test_exchange_auto_rule_and_argument_checks():
    """exchange="auto" sends a step as flagged packets up to PACKET_BYTES_PER_PEER bytes of rows per peer
    and as stores + barrier above (config 2 at 2 GPUs: 64 rows of 16 heads x 128 dims x 2 B = 256 KB ->
    packets, 128 rows -> barrier); a fixed mode ignores the size; a bad mode is refused."""
    from importlib import import_module

    sharding = import_module(PACKAGE + ".sharding")
    p = object.__new__(sharding.PeerOutputs)  # the rule alone: no IPC allocation
    p._row_bytes = 16 * 128 * 2
    p.exchange = "auto"
    assert sharding.PACKET_BYTES_PER_PEER == 384 << 10
    assert p.use_packets(64) and not p.use_packets(128)
    p.exchange = "packets"
    assert p.use_packets(1 << 20)
    p.exchange = "barrier"
    assert not p.use_packets(1)
    own = not dist.is_initialized()
    if own:
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    try:
        with pytest.raises(ValueError, match="exchange"):
            sharding.KVHeadShardedBackend(transport="p2p", exchange="fast")
        assert sharding.KVHeadShardedBackend(transport="p2p").exchange == "auto"
    finally:
        if own:
            dist.destroy_process_group()
