"""The output gather of KV-head sharding on the GPU: attention rows stored into several destinations
(mlb_out_targets) equal the plain output bit for bit in each; the reduction carrying the gather fills
every destination; `PeerOutputs` over a one-rank group (IPC allocation, slot views, barrier, the packet
exchange); the flag barrier and the packet exchange advance their device epochs under CUDA-graph replay,
and their bounded waits run out and report MLB_DEV_WAIT_TIMEOUT when a peer never arrives (a flag or a
packet nothing writes).
With two or more GPUs visible, `peer_worker.py` runs under torchrun and checks the p2p gather against the
NCCL all-gather and the oracle."""

from __future__ import annotations

import ctypes
import os
import socket
import subprocess
import sys

import pytest
import torch

import cases
from conftest import REPO
from paged_helpers import assert_close, bits, device_case, oracle_forward

pytestmark = pytest.mark.gpu


def _setup(mlb, case, dtype, dev, ppu):
    t = device_case(case, dtype, dev)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], case.bs, dev)
    mlb.kv_append(t["k_pool"], t["v_pool"], meta.slot_mapping, t["k"], t["v"])
    plan = mlb.plan_attention(meta.query_start_loc, meta.seq_lens, meta.block_tables_i32.shape[1], case.h, case.hkv,
                              dev, pages_per_unit=ppu)
    return t, meta, plan


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=str)
def test_rows_reach_every_destination(mlb, cuda, dtype):
    case = cases.boundaries(6, 32, 8, 128)
    t, meta, plan = _setup(mlb, case, dtype, cuda, ppu=2)
    split = plan.units_host[:, 4] >= 0
    assert split.any() and (~split).any(), "the case must have split and unsplit units"
    ws = mlb.Workspace()
    args = (t["q"], t["k_pool"], t["v_pool"], meta.block_tables_i32, meta.seq_lens_i32, meta.qo_indptr, plan, ws)
    ref = mlb.paged_attention(*args)
    n, h, dh = ref.shape
    # three destinations laid out as rank 1 of 2 would see them: [n, 2h, dh], this call's heads at offset h
    bufs = [torch.full((n, 2 * h, dh), float("nan"), dtype=dtype, device=cuda) for _ in range(3)]
    tg = mlb.ops.out_targets([b.data_ptr() for b in bufs], h, 2 * h * dh, dh)
    assert mlb.paged_attention(*args, targets=tg) is None
    for b in bufs:
        assert torch.equal(bits(b[:, h:].contiguous()), bits(ref))
        assert torch.isnan(b[:, :h]).all()  # the other rank's heads are not touched
    assert_close(ref, oracle_forward(case, dtype)[0], dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=str)
def test_reduce_gather_fills_every_destination(mlb, cuda, dtype):
    """mlb_splitk_reduce_gather on one GPU: destination 0 is this rank's buffer (the attention kernel's
    unsplit rows go only there), destinations 1 and 2 stand for peers; all three end equal to the plain
    output.  Also with a plan that split nothing (the reduction then only copies rows)."""
    for ppu in (2, 0):
        case = cases.boundaries(6, 32, 8, 128) if ppu else cases.llama_decode(5, 3, 20, 120)
        t, meta, plan = _setup(mlb, case, dtype, cuda, ppu=ppu)
        assert (plan.num_partial_rows > 0) == bool(ppu)
        ws = mlb.Workspace()
        args = (t["q"], t["k_pool"], t["v_pool"], meta.block_tables_i32, meta.seq_lens_i32, meta.qo_indptr, plan)
        ref = mlb.paged_attention(*args, ws)
        n, h, dh = ref.shape
        bufs = [torch.full((n, 2 * h, dh), float("nan"), dtype=dtype, device=cuda) for _ in range(3)]
        ptrs = [b.data_ptr() for b in bufs]
        mlb.ops.attention_partials(*args, ws, targets=mlb.ops.out_targets(ptrs[:1], h, 2 * h * dh, dh))
        mlb.ops.splitk_reduce_gather(plan, ws, mlb.ops.out_targets(ptrs, h, 2 * h * dh, dh), 0, dtype, dh, cuda)
        for b in bufs:
            assert torch.equal(bits(b[:, h:].contiguous()), bits(ref))
            assert torch.isnan(b[:, :h]).all()


def _barrier(L, flags, rank, world, epoch, timeout_ns, err):
    arr = (ctypes.c_void_p * world)(*[f.data_ptr() for f in flags])
    L.check(L.lib().mlb_peer_barrier(arr, rank, world, epoch.data_ptr(), timeout_ns, err.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream), "peer_barrier")


def test_barrier_alone_advances_its_epoch_under_graph_replay(mlb, cuda):
    L = mlb._lib
    flags = [torch.zeros(8, dtype=torch.int32, device=cuda)]
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for _ in range(3):
        _barrier(L, flags, 0, 1, epoch, 0, err)
    torch.cuda.synchronize()
    assert epoch.item() == 3 and flags[0][0].item() == 3 and err.item() == 0
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(2):
                _barrier(L, flags, 0, 1, epoch, 0, err)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(4):
        g.replay()
    torch.cuda.synchronize()
    assert epoch.item() == 11 and flags[0][0].item() == 11 and err.item() == 0


def test_barrier_wait_runs_out_when_a_peer_never_arrives(mlb, cuda):
    """Rank 0 of 2 with both flag arrays local: nothing ever raises rank 1's word in rank 0's array, so the
    wait must give up after its limit (50 ms here) and say so in the error word."""
    L = mlb._lib
    flags = [torch.zeros(8, dtype=torch.int32, device=cuda) for _ in range(2)]
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _barrier(L, flags, 0, 2, epoch, 50_000_000, err)
    torch.cuda.synchronize()
    assert err.item() & L.DEV_WAIT_TIMEOUT
    assert flags[0][0].item() == 1 and flags[1][0].item() == 1 and flags[0][1].item() == 0
    assert epoch.item() == 1


def test_peer_outputs_single_rank(mlb, cuda):
    import torch.distributed as dist

    sharding = __import__(mlb.__name__ + ".sharding", fromlist=["PeerOutputs"])
    own_group = not dist.is_initialized()
    if own_group:
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    try:
        case = cases.mixed_step(4, 32, 8, 128)
        t, meta, plan = _setup(mlb, case, torch.bfloat16, cuda, ppu=3)
        ws = mlb.Workspace()
        args = (t["q"], t["k_pool"], t["v_pool"], meta.block_tables_i32, meta.seq_lens_i32, meta.qo_indptr, plan, ws)
        ref = mlb.paged_attention(*args)
        n, h, dh = ref.shape
        peers = sharding.PeerOutputs(n + 5, h, dh, torch.bfloat16, cuda, slots=2)
        for slot in (0, 1, 0):
            peers.output(slot, n).fill_(float("nan"))
            mlb.paged_attention(*args, targets=peers.targets(slot, 0))
            peers.barrier()
            assert torch.equal(bits(peers.output(slot, n)), bits(ref))
            peers.output(slot, n).fill_(float("nan"))
            mlb.ops.attention_partials(*args[:-1], ws, targets=peers.local_targets(slot, 0))
            mlb.ops.splitk_reduce_gather(plan, ws, peers.targets(slot, 0), peers.self_dest, torch.bfloat16, dh, cuda)
            peers.barrier()
            assert torch.equal(bits(peers.output(slot, n)), bits(ref))
        peers.raise_errors()
        with pytest.raises(ValueError, match="capacity"):
            peers.output(0, n + 6)
        peers.close()
    finally:
        if own_group:
            dist.destroy_process_group()


def _exchange(L, dt, plan, ws, out, n_heads, dh, areas, capacity, rank, world, state, timeout_ns, err):
    po = plse = None
    if plan.num_partial_rows:
        po, plse = ws.get(plan.num_partial_rows, plan.num_heads, dh, out.device)
    arr = (ctypes.c_void_p * len(areas))(*[a.data_ptr() for a in areas])
    L.check(L.lib().mlb_splitk_reduce_exchange(
        0 if po is None else po.data_ptr(), 0 if plse is None else plse.data_ptr(), plan.num_partial_rows,
        plan.reduce_rows.data_ptr(), plan.reduce_chunks.data_ptr(), plan.tokens_per_tile, plan.num_tokens,
        plan.num_heads, dh, dt, out.data_ptr(), out.stride(0), out.stride(1), arr, capacity, rank, world,
        state.data_ptr(), timeout_ns, err.data_ptr(), torch.cuda.current_stream().cuda_stream), "splitk_reduce_exchange")


def test_exchange_single_rank_finishes_rows_and_advances_its_epoch(mlb, cuda):
    """One rank: the exchange has no peer to send to or wait for; it finishes the split rows into the own
    buffer (bit-equal to the plain output) and advances its epoch once per call, also under graph replay."""
    L = mlb._lib
    case = cases.boundaries(6, 32, 8, 128)
    t, meta, plan = _setup(mlb, case, torch.bfloat16, cuda, ppu=2)
    assert plan.num_partial_rows > 0
    ws = mlb.Workspace()
    args = (t["q"], t["k_pool"], t["v_pool"], meta.block_tables_i32, meta.seq_lens_i32, meta.qo_indptr, plan, ws)
    ref = mlb.paged_attention(*args)
    n, h, dh = ref.shape
    out = torch.full((n, h, dh), float("nan"), dtype=torch.bfloat16, device=cuda)
    areas = [torch.zeros(n * h * dh * 2 * 2 // 8, dtype=torch.int64, device=cuda) for _ in range(2)]
    state = torch.zeros(2, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    tg = mlb.ops.out_targets([out.data_ptr()], 0, h * dh, dh)

    def step():
        mlb.ops.attention_partials(*args, targets=tg)
        _exchange(L, L.MLB_BF16, plan, ws, out, h, dh, areas, n, 0, 1, state, 0, err)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    assert torch.equal(bits(out), bits(ref)) and state.tolist() == [3, 0] and err.item() == 0
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            step()
            step()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(4):
        g.replay()
    torch.cuda.synchronize()
    assert state.tolist() == [11, 0] and err.item() == 0
    assert torch.equal(bits(out), bits(ref))


def test_exchange_wait_runs_out_when_a_peer_never_sends(mlb, cuda):
    """Rank 0 of 2 with every packet area local: rank 0's packets land in "rank 1's" area with epoch 1 (area
    1 = the epoch's parity), nothing ever writes rank 1's packets into rank 0's area, so the wait gives up
    after its limit (50 ms here) and says so in the error word; the epoch still advances."""
    L = mlb._lib
    case = cases.llama_decode(5, 3, 20, 120)
    t, meta, plan = _setup(mlb, case, torch.bfloat16, cuda, ppu=0)
    ws = mlb.Workspace()
    args = (t["q"], t["k_pool"], t["v_pool"], meta.block_tables_i32, meta.seq_lens_i32, meta.qo_indptr, plan, ws)
    n, h, dh = t["q"].shape
    out = torch.zeros((n, 2 * h, dh), dtype=torch.bfloat16, device=cuda)
    words = dh * 2 // 4  # 32-bit words per row
    areas = [torch.zeros(n * 2 * h * words, dtype=torch.int64, device=cuda) for _ in range(4)]  # [area][rank]
    state = torch.zeros(2, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    mlb.ops.attention_partials(*args, targets=mlb.ops.out_targets([out.data_ptr()], 0, 2 * h * dh, dh))
    _exchange(L, L.MLB_BF16, plan, ws, out, h, dh, areas, n, 0, 2, state, 50_000_000, err)
    torch.cuda.synchronize()
    assert err.item() & L.DEV_WAIT_TIMEOUT
    assert state.tolist() == [1, 0]
    sent = areas[1 * 2 + 1].view(n, 2, h, words)  # area 1 of rank 1: rank 0's rows at sender index 0
    assert (sent[:, 0] >> 32 == 1).all() and (sent[:, 1] == 0).all()
    mine = out[:, :h].contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF  # rank 0's finished rows
    assert torch.equal(sent[:, 0] & 0xFFFFFFFF, mine)
    assert (areas[0] == 0).all() and (areas[1] == 0).all() and (areas[2] == 0).all()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_p2p_gather_matches_nccl_on_two_gpus():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(REPO / "tests" / "peer_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env={**os.environ, "NCCL_NVLS_ENABLE": "0"})
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("peer gather ok") == 2
