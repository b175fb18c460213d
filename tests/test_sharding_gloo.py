"""Multi-rank host logic on CPU (gloo, world_size 2, and 4 for the gather): the
head-shard plan, the all-gather of o, a head-sharded prefill (oracle as the per-rank compute, the
CUDA kernel is covered by the GPU tests) equal to the unsharded result, and
failure detection when a rank dies before the collective."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gdn_18646_b200 import sharding as SH


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def test_head_shard_plan():
    shards = [SH.head_shard(32, r, 4) for r in range(4)]
    assert [(s.h0, s.h1) for s in shards] == [(0, 8), (8, 16), (16, 24), (24, 32)]
    with pytest.raises(ValueError):
        SH.head_shard(30, 0, 4)
    with pytest.raises(ValueError):          # 2 heads per rank would cut groups of 4
        SH.head_shard(8, 0, 4, Hqk=2)
    assert SH.head_shard(32, 1, 2, Hqk=16).count == 16
    sl = [SH.batch_shard(10, r, 4) for r in range(4)]
    assert [(s.start, s.stop) for s in sl] == [(0, 3), (3, 6), (6, 8), (8, 10)]


@pytest.mark.parametrize("T", [1, 63, 64, 65, 1000, 4096, 32768, 70001])
@pytest.mark.parametrize("w", [0, 64, 1000, 4096])
def test_window_plan(T, w):
    for ladder in (True, False):
        plan = SH.window_plan(T, w, ladder)
        assert plan[0][0] == 0 and sum(tw for _, tw in plan) == T
        assert all(t0 + tw == nxt for (t0, tw), (nxt, _) in zip(plan, plan[1:]))   # contiguous
        assert all(t0 % 64 == 0 for t0, _ in plan)                                  # chunk-aligned starts
        wt = -(-w // 64) * 64 if w else None
        if wt:
            assert max(tw for _, tw in plan) <= wt
        if ladder and len(plan) > 1:
            assert plan[-1][1] <= 64                                                # a one-chunk tail
    assert [tw for _, tw in SH.window_plan(32768, 4096, False)] == [4096] * 8
    assert [tw for _, tw in SH.window_plan(32768, 4096, True)] == [4096] * 7 + [2048, 1024, 512, 256, 128, 64, 64]
    with pytest.raises(ValueError):
        SH.window_plan(0)
    with pytest.raises(ValueError):
        SH.window_plan(64, -1)


def _gather_worker(rank, world, port, q):
    _init(rank, world, port)
    try:
        full = torch.arange(2 * 3 * 8 * 4, dtype=torch.float32).reshape(2, 3, 8, 4)
        sh = SH.head_shard(8, rank, world)
        got = SH.gather_heads(SH.shard_heads(full, sh, 2), sh)
        q.put((rank, bool(torch.equal(got, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gather_heads_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(60)
    assert res == {r: True for r in range(world)}


def _sharded_oracle_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import gdn_oracle as O
    _init(rank, world, port)
    try:
        inp = O.make_prefill_inputs(11, 1, 128, 4, 64, 64, state_std=0.02, layout="bthd", Hqk=2)
        sh = SH.head_shard(4, rank, world, Hqk=2)
        g = 4 // 2
        qh = np.swapaxes(inp["q"], 1, 2)[:, sh.h0 // g:sh.h1 // g]
        kh = np.swapaxes(inp["k"], 1, 2)[:, sh.h0 // g:sh.h1 // g]
        vh = np.swapaxes(inp["v"], 1, 2)[:, sh.h0:sh.h1]
        o, S = O.prefill(O.expand_qk_heads(qh, sh.count), O.expand_qk_heads(kh, sh.count), vh,
                         inp["A_log"][sh.h0:sh.h1], inp["a"][:, sh.h0:sh.h1], 0.0, inp["b"][:, sh.h0:sh.h1],
                         inp["mask"], state_in=inp["state_in"][:, sh.h0:sh.h1], scale=inp["scale"], chunk_size=64)
        o_full = SH.gather_heads(torch.from_numpy(np.ascontiguousarray(np.swapaxes(o, 1, 2))), sh)
        q.put((rank, o_full.numpy(), S))
    finally:
        dist.destroy_process_group()


def test_sharded_prefill_equals_unsharded_gloo():
    from oracle import gdn_oracle as O
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_oracle_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (o, S) for r, o, S in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(60)
    inp = O.make_prefill_inputs(11, 1, 128, 4, 64, 64, state_std=0.02, layout="bthd", Hqk=2)
    o_ref, S_ref = O.prefill(O.expand_qk_heads(np.swapaxes(inp["q"], 1, 2), 4),
                             O.expand_qk_heads(np.swapaxes(inp["k"], 1, 2), 4), np.swapaxes(inp["v"], 1, 2),
                             inp["A_log"], inp["a"], 0.0, inp["b"], inp["mask"], state_in=inp["state_in"],
                             scale=inp["scale"], chunk_size=64)
    for r in (0, 1):
        np.testing.assert_allclose(res[r][0], np.swapaxes(o_ref, 1, 2), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(np.concatenate([res[0][1], res[1][1]], 1), S_ref, rtol=1e-5, atol=1e-6)


def _failing_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    try:
        if rank == 1:
            raise RuntimeError("rank 1 failed before the collective")
        sh = SH.head_shard(4, rank, world)
        SH.gather_heads(torch.zeros(1, 2, 2, 3), sh)
        q.put((rank, "no error"))
    except Exception as e:              # the survivor sees the failure as an exception
        q.put((rank, type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_failure_surfaces_as_error_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    assert res[1] == "RuntimeError"
    assert res[0] != "no error"
