"""The sequence-sharded far memory on CPU ranks (gloo, world size 2).

Each rank holds one contiguous chunk of the side cache (ShardPlan), computes the partial of its
chunk (here with the oracle, standing in for the GPU far read + combine kernels), the partials
are exchanged with the same all-gather code the GPU path uses (fold_b200.shard), and the merge of
all partials must equal the unsharded read. A rank that fails before the exchange must make the
other rank's collective fail within the process-group timeout instead of hanging.
"""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fold_b200.shard import ShardPlan, exchange_partials, gather_handles, pack_partial, unpack_partials
from oracle import fold_oracle as fo


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def problem(seed=3):
    rng = np.random.default_rng(seed)
    n, hq, hkv, d, W = 6, 8, 2, 32, 40
    length = 1500
    hist = length - n
    k = rng.standard_normal((length, hkv, d))
    v = rng.standard_normal((length, hkv, d))
    qf = rng.standard_normal((n, hq, d))
    return dict(n=n, hq=hq, hkv=hkv, d=d, W=W, length=length, hist=hist, k=k, v=v, qf=qf, scale=0.25)


def rank_partial(p, plan):
    lim = fo.far_row_limits(p["hist"], p["W"], p["n"], p["n"])
    lo, held = plan.pos_lo, plan.held
    lim_local = np.minimum(lim, lo + held)
    return fo.far_read(p["qf"], p["k"][lo:lo + held], p["v"][lo:lo + held], lim_local, p["scale"], key_lo=lo)


def worker(rank, world, port, mode, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
        p = problem()
        plan = ShardPlan.even(p["length"], world, rank)
        o, lse = rank_partial(p, plan)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the exchange")
        if mode == "handles":
            mine = bytes((rank * 37 + i) % 256 for i in range(64))
            out_q.put((rank, "ok", gather_handles(mine)))
            return
        o_all, lse_all = exchange_partials(torch.from_numpy(o).float(), torch.from_numpy(lse).float())
        out_q.put((rank, "ok", (o_all.numpy().astype(np.float64), lse_all.numpy().astype(np.float64))))
    except Exception as e:  # reported to the parent, which decides what was expected
        out_q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc(limit=2)}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def run(world, mode, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, mode, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    results = {}
    for _ in range(world):
        rank, status, payload = q.get(timeout=timeout)
        results[rank] = (status, payload)
    for pr in procs:
        pr.join(timeout=timeout)
        if pr.is_alive():
            pr.kill()
    return results


@pytest.mark.parametrize("kind", ["even", "for_far"])
def test_shard_plan_covers_every_position_once(kind):
    for length, world in ((131072 + 2000, 8), (1500, 2), (300, 4), (262144, 3)):
        if kind == "even":
            plans = [ShardPlan.even(length, world, r) for r in range(world)]
        else:
            plans = [ShardPlan.for_far(length, 2048 if length > 4096 else 40, 10, world, r) for r in range(world)]
        covered = np.zeros(length, dtype=int)
        for p in plans:
            assert p.pos_lo % 256 == 0 and p.chunk % 256 == 0
            covered[p.pos_lo:p.pos_lo + p.held] += 1
        assert np.all(covered == 1)
        for pos in (0, length // 2, length - 1):
            p = plans[plans[0].owner(pos)]
            assert p.pos_lo <= pos < p.pos_lo + p.held


def test_far_plan_balances_the_far_keys():
    length, W, B = 131072 + 1100, 2048, 10
    far = length - W - B
    for world in (2, 4, 8):
        plans = [ShardPlan.for_far(length, W, B, world, r) for r in range(world)]
        keys = [max(0, min(p.pos_lo + p.held, far) - p.pos_lo) for p in plans]
        assert sum(keys) == far
        assert max(keys) - min(keys) <= world * 256  # whole pages: the last rank takes the rest


def test_pack_unpack_round_trip():
    o = torch.randn(3, 4, 8)
    lse = torch.randn(4, 3)
    buf = torch.cat([pack_partial(o, lse), pack_partial(o + 1, lse - 1)])
    oa, la = unpack_partials(buf, 2, 3, 4, 8)
    assert torch.equal(oa[0], o) and torch.equal(oa[1], o + 1) and torch.equal(la[1], lse - 1)


def test_sharded_exchange_matches_unsharded_read():
    results = run(2, "ok")
    assert all(s == "ok" for s, _ in results.values()), results
    p = problem()
    lim = fo.far_row_limits(p["hist"], p["W"], p["n"], p["n"])
    o_ref, lse_ref = fo.far_read(p["qf"], p["k"], p["v"], lim, p["scale"])
    for rank in (0, 1):
        o_all, lse_all = results[rank][1]
        o, lse = fo.combine(o_all, lse_all)
        np.testing.assert_allclose(o, o_ref, atol=1e-5)
        fin = np.isfinite(lse_ref)
        assert np.array_equal(np.isfinite(lse), fin)
        np.testing.assert_allclose(lse[fin], lse_ref[fin], atol=1e-5)


@pytest.mark.timeout(120)
def test_failed_rank_makes_the_exchange_fail_not_hang():
    results = run(2, "fail")
    assert results[1][0] == "error" and "fails before the exchange" in results[1][1]
    assert results[0][0] == "error", results[0]


def test_exchange_handles_are_gathered_in_rank_order():
    """The peer exchange's setup shares every rank's 64-byte IPC handle; every rank must receive all
    of them, concatenated in rank order."""
    world = 2
    results = run(world, "handles")
    want = b"".join(bytes((r * 37 + i) % 256 for i in range(64)) for r in range(world))
    for r in range(world):
        assert results[r] == ("ok", want)
