"""The peer exchange kernel (fold_exchange_merge) on one GPU, as a group of one rank: its combine
of the split partials, its push/flag/wait protocol (local here) and its merge must give exactly
the merge kernel's output, and match the oracle's combine + merge; repeated launches and graph
replays advance the device epoch without a host input. The multi-rank protocol runs in
test_gpu_shard.py when 2 GPUs are present."""
import numpy as np
import pytest
import torch

from fold_b200 import kernels
from fold_b200.errors import FoldError
from fold_b200.shard import PeerExchange
from oracle import fold_oracle as fo
from tests.helpers import OUT_ATOL, to64

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)


def partials(seed, S, n, hq, hd, empty_every=5):
    g = torch.Generator().manual_seed(seed)
    o = torch.randn((S, n, hq, hd), generator=g)
    lse = torch.randn((S, hq, n), generator=g) * 3 + 8
    lse.view(-1)[::empty_every] = -float("inf")  # empty splits carry no mass
    o_l = torch.randn((n, hq, hd), generator=g).to(torch.bfloat16)
    lse_l = torch.randn((hq, n), generator=g) + 6
    return [t.cuda() for t in (o, lse, o_l, lse_l)]


@pytest.mark.parametrize("S,n,hq,hd,hist", [(18, 10, 32, 128, 131062), (37, 16, 16, 256, 262128), (5, 3, 4, 64, 2100),
                                            (7, 10, 8, 128, 2050)])
def test_single_rank_exchange_equals_merge_kernel(S, n, hq, hd, hist):
    W, B, alpha = 2048, n, 2.0
    o, lse, o_l, lse_l = partials(S + n, S, n, hq, hd)
    qsl = torch.tensor([0, n], dtype=torch.int32, device="cuda")
    seq = torch.tensor([hist + n], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = torch.empty((n, hq, hd), dtype=torch.bfloat16, device="cuda")
    kernels.merge(o_l, lse_l, o, lse, want, qsl, seq, window=W, block=B, alpha=alpha)
    ex = PeerExchange(n=n, hq=hq, hd=hd)
    try:
        got = torch.empty_like(want)
        ex.merge(o, lse, o_l, lse_l, got, qsl, seq, window=W, block=B, alpha=alpha, err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(got, want)
        o_f, lse_f = fo.combine(to64(o), to64(lse))
        ref = fo.merge(to64(o_l), to64(lse_l), o_f, lse_f, hist, W, B, alpha)
        assert np.abs(to64(got) - ref).max() <= OUT_ATOL
    finally:
        ex.close()


def test_exchange_epochs_advance_across_calls_and_graph_replays():
    S, n, hq, hd, W, B, hist = 18, 10, 32, 128, 2048, 10, 50000
    qsl = torch.tensor([0, n], dtype=torch.int32, device="cuda")
    seq = torch.tensor([hist + n], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    steps = [partials(100 + i, S, n, hq, hd) for i in range(3)]
    want = []
    for o, lse, o_l, lse_l in steps:
        w = torch.empty((n, hq, hd), dtype=torch.bfloat16, device="cuda")
        kernels.merge(o_l, lse_l, o, lse, w, qsl, seq, window=W, block=B, alpha=2.0)
        want.append(w)
    ex = PeerExchange(n=n, hq=hq, hd=hd)
    outs = [torch.empty((n, hq, hd), dtype=torch.bfloat16, device="cuda") for _ in steps]
    try:
        for _ in range(3):  # eager calls: epochs 1..9
            for (o, lse, o_l, lse_l), out in zip(steps, outs):
                ex.merge(o, lse, o_l, lse_l, out, qsl, seq, window=W, block=B, alpha=2.0, err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert all(torch.equal(a, b) for a, b in zip(outs, want))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for (o, lse, o_l, lse_l), out in zip(steps, outs):
                ex.merge(o, lse, o_l, lse_l, out, qsl, seq, window=W, block=B, alpha=2.0, err=err)
        for out in outs:
            out.zero_()
        for _ in range(5):  # 15 more epochs, both parities, no host input
            graph.replay()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert all(torch.equal(a, b) for a, b in zip(outs, want))
        del graph
    finally:
        ex.close()


def test_exchange_rejects_a_larger_step_than_created_for():
    ex = PeerExchange(n=4, hq=8, hd=128)
    try:
        o, lse, o_l, lse_l = partials(1, 3, 6, 8, 128)
        qsl = torch.tensor([0, 6], dtype=torch.int32, device="cuda")
        seq = torch.tensor([9000], dtype=torch.int32, device="cuda")
        with pytest.raises(FoldError, match="larger"):
            ex.merge(o, lse, o_l, lse_l, torch.empty_like(o_l), qsl, seq, window=2048, block=6, alpha=2.0)
    finally:
        ex.close()


def far_case(seed, n, hq, hkv, hd, hist):
    from fold_b200.attention import FoldWorkspace
    from fold_b200.rope import default_inv_freq
    from tests.helpers import side_from

    rng = np.random.default_rng(seed)
    W, B = 2048, n
    seq = hist + n
    k = rng.standard_normal((seq, hkv, hd), dtype=np.float32)
    v = rng.standard_normal((seq, hkv, hd), dtype=np.float32)
    q = torch.from_numpy(rng.standard_normal((n, hq, hd), dtype=np.float32)).cuda().to(torch.bfloat16)
    dummy = torch.zeros((1, hkv, 16, 2 * hd), device="cuda", dtype=torch.bfloat16)
    ws = FoldWorkspace(dummy, W, B, seq, inv_freq=default_inv_freq(500000.0, hd, "cuda"), far_distance=W + B,
                       num_heads=hq)
    ws.side = side_from(k, v, ws.side_pages)
    o_l = torch.from_numpy(rng.standard_normal((n, hq, hd), dtype=np.float32)).cuda().to(torch.bfloat16)
    lse_l = torch.from_numpy(rng.standard_normal((hq, n), dtype=np.float32) + 6).cuda()
    qsl = torch.tensor([0, n], dtype=torch.int32, device="cuda")
    seq_t = torch.tensor([seq], dtype=torch.int32, device="cuda")
    return ws, q, o_l, lse_l, qsl, seq_t


@pytest.mark.parametrize("n,hq,hkv,hd,hist", [(10, 32, 8, 128, 40000), (8, 32, 8, 128, 2060), (3, 8, 2, 256, 9000),
                                              (1, 4, 4, 128, 5000)])
def test_single_rank_far_read_exchange_equals_far_read_and_merge(n, hq, hkv, hd, hist, far_kernel):
    """fold_far_read_exchange with a one-rank exchange (far read + merge in one launch) against
    fold_far_read followed by fold_merge: the same far partials, the same merge up to the order of
    the split combine, so within one bf16 rounding."""
    ws, q, o_l, lse_l, qsl, seq = far_case(hist + n, n, hq, hkv, hd, hist)
    scale = hd ** -0.5
    want = torch.empty((n, hq, hd), dtype=torch.bfloat16, device="cuda")
    o_part, lse_part = ws.read_far(q, qsl, seq, scale)
    kernels.merge(o_l, lse_l, o_part, lse_part, want, qsl, seq, window=ws.window, block=ws.block, alpha=ws.alpha)
    ex = PeerExchange(n=n, hq=hq, hd=hd)
    try:
        got = torch.empty_like(want)
        ex.read_merge(ws, q, qsl, seq, scale, o_l, lse_l, got)
        torch.cuda.synchronize()
        ws.check()
        diff = (got.float() - want.float()).abs()
        assert float(diff.max()) <= 2 ** -7 * float(want.float().abs().max())
        # repeated launches and graph replays advance the epochs and reset the split counters
        graph = torch.cuda.CUDAGraph()
        outs = [torch.empty_like(want) for _ in range(3)]
        with torch.cuda.graph(graph):
            for o in outs:
                ex.read_merge(ws, q, qsl, seq, scale, o_l, lse_l, o)
        for _ in range(4):
            graph.replay()
        torch.cuda.synchronize()
        ws.check()
        assert all(torch.equal(o, got) for o in outs)
        del graph
    finally:
        ex.close()


def _silent_peer_worker(rank, port, q):
    """Rank 0 merges through a two-rank exchange whose rank 1 never takes the step (both ranks on
    cuda:0; rank 1 only maps its region and waits on the host). Rank 0's wait for rank 1's record
    runs out after its bounded limit, the kernel records the timeout and merges what it has."""
    import os
    import time

    import torch.distributed as dist

    from fold_b200.errors import DEVERR_TIMEOUT
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    ex = None
    try:
        dist.init_process_group("gloo", rank=rank, world_size=2)
        S, n, hq, hd, W, B, hist = 6, 4, 8, 128, 2048, 4, 9000
        ex = PeerExchange(n=n, hq=hq, hd=hd)
        result = None
        if rank == 0:
            o, lse, o_l, lse_l = partials(7, S, n, hq, hd)
            qsl = torch.tensor([0, n], dtype=torch.int32, device="cuda")
            seq = torch.tensor([hist + n], dtype=torch.int32, device="cuda")
            err = torch.zeros(1, dtype=torch.int32, device="cuda")
            out = torch.empty((n, hq, hd), dtype=torch.bfloat16, device="cuda")
            times, words = [], []
            for _ in range(2):
                err.zero_()
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                ex.merge(o, lse, o_l, lse_l, out, qsl, seq, window=W, block=B, alpha=2.0, err=err)
                torch.cuda.synchronize()
                times.append(time.perf_counter() - t0)
                words.append(int(err.item()))
            # the context is still usable: the plain merge of the same partials runs and agrees
            want = torch.empty_like(out)
            kernels.merge(o_l, lse_l, o, lse, want, qsl, seq, window=W, block=B, alpha=2.0)
            torch.cuda.synchronize()
            result = (times, words, DEVERR_TIMEOUT, to64(out), to64(want))
        ex.close()  # both ranks meet here, after rank 0's launches have finished
        ex = None
        q.put((rank, "ok", result))
    except Exception as e:
        q.put((rank, "error", repr(e)))
    finally:
        if ex is not None:
            ex.close()
        if dist.is_initialized():
            dist.destroy_process_group()


def test_exchange_wait_runs_out_when_a_peer_never_merges():
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_silent_peer_worker, args=(r, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = dict((r, (st, x)) for r, st, x in (q.get(timeout=300) for _ in range(2)))
    for pr in procs:
        pr.join(timeout=60)
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    times, words, timeout_bit, out, want = res[0][1]
    # first launch: the wait gives up after its 2 s limit; second: the exchange is poisoned and
    # the launch does not wait at all
    assert all(w & timeout_bit for w in words), words
    assert 1.5 <= times[0] <= 30.0, times
    assert times[1] < 1.0, times
    # with the peer's partial missing, the output is this rank's own merge
    np.testing.assert_array_equal(out, want)
