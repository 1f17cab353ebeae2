"""Multi-rank host logic on CPU (gloo, world size 2): view sharding, the
flattened shared-gradient all-reduce, max-over-ranks timing, and failure
detection when a rank dies before the collective (the survivor's collective
ends with an error instead of hanging)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=20):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_allreduce(rank, world, port, q):
    import sys
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "mlx-swift-diffrast_b200"))
    from diffrast import dist as D
    try:
        _init(rank, world, port)
        lo, hi, tot = D.view_range(32, rank, world, weak=True)
        slo, shi, stot = D.view_range(256, rank, world, weak=False)
        g1 = torch.full((5, 4), float(rank + 1))
        g2 = torch.arange(7, dtype=torch.float32) * (rank + 1)
        D.allreduce_grads([g1, None, g2])
        m = D.max_over_ranks(float(rank) + 0.5)
        q.put((rank, (lo, hi, tot), (slo, shi, stot), g1.tolist(), g2.tolist(), m))
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        q.put((rank, "error", repr(e)))


def _worker_gradsync(rank, world, port, q):
    import sys
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "mlx-swift-diffrast_b200"))
    from diffrast import dist as D
    try:
        _init(rank, world, port)
        a = torch.ones(4, requires_grad=True)
        b = torch.full((3,), 2.0, requires_grad=True)
        sync = D.GradSync([a, b])
        for step in range(2):  # the hooks stay registered across steps
            a.grad = None
            b.grad = None
            loss = (a * (rank + 1)).sum() + (b * b * (rank + 1)).sum()
            loss.backward()
            sync.finish()
        q.put((rank, a.grad.tolist(), b.grad.tolist()))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, "error", repr(e)))


def _worker_gradsync_micro(rank, world, port, q):
    """Two backward calls per step (micro-batches), as the sharded cfg5 chain
    runs them: the all-reduce must start once, after the last backward."""
    import sys
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "mlx-swift-diffrast_b200"))
    from diffrast import dist as D
    try:
        _init(rank, world, port)
        a = torch.ones(4, requires_grad=True)
        b = torch.full((3,), 2.0, requires_grad=True)
        sync = D.GradSync([a, b])
        launched = []
        for step in range(2):
            a.grad = None
            b.grad = None
            for micro in range(2):
                sync.arm(micro == 1)
                # micro-batch k contributes (k + 1) * (rank + 1) to d/da
                loss = (a * (micro + 1) * (rank + 1)).sum() + (b * b * (rank + 1)).sum()
                loss.backward()
                launched.append(len(sync.handles))
            sync.finish()
        q.put((rank, a.grad.tolist(), b.grad.tolist(), launched))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, "error", repr(e)))


def _worker_dead_peer(rank, world, port, q):
    import time
    import torch
    import torch.distributed as dist
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush the message before dying
            os._exit(0)  # dies between steps, before the collective
        time.sleep(0.5)
        t0 = time.time()
        try:
            dist.all_reduce(torch.ones(3))
            q.put((rank, "no-error", time.time() - t0))
        except Exception as e:
            q.put((rank, "error", time.time() - t0, type(e).__name__))
    except Exception as e:
        q.put((rank, "init-error", repr(e)))


def _run(target, world=2, timeout=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = []
    for _ in range(world):
        out.append(q.get(timeout=timeout))
    for p in ps:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_allreduce_and_sharding_two_ranks():
    res = _run(_worker_allreduce)
    for r in res:
        assert r[1] != "error", r
    (r0, w0, s0, g1_0, g2_0, m0), (r1, w1, s1, g1_1, g2_1, m1) = res
    assert w0 == (0, 32, 64) and w1 == (32, 64, 64)          # weak: disjoint global views
    assert s0 == (0, 128, 256) and s1 == (128, 256, 256)     # strong: 256 views split
    assert g1_0 == g1_1 == [[3.0] * 4] * 5                   # 1 + 2
    assert g2_0 == g2_1 == [3.0 * i for i in range(7)]
    assert m0 == m1 == 1.5


def test_dead_rank_makes_the_survivor_fail_not_hang():
    res = _run(_worker_dead_peer)
    d = {r[0]: r for r in res}
    assert d[1][1] == "left"
    assert d[0][1] == "error", d[0]
    assert d[0][2] < 60


def test_view_range_rejects_uneven_strong_split():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "mlx-swift-diffrast_b200"))
    from diffrast import dist as D
    with pytest.raises(ValueError):
        D.view_range(10, 0, 3, weak=False)


def test_gradsync_sums_gradients_as_they_finish():
    res = _run(_worker_gradsync)
    for r in res:
        assert r[1] != "error", r
    # d/da = rank + 1 summed over ranks = 3; d/db = 2 b (rank + 1) summed = 4 * 3 = 12
    assert res[0][1] == res[1][1] == [3.0] * 4
    assert res[0][2] == res[1][2] == [12.0] * 3


def test_gradsync_reduces_once_after_the_last_micro_batch():
    res = _run(_worker_gradsync_micro)
    for r in res:
        assert r[1] != "error", r
    # d/da per rank = (1 + 2)(rank + 1), summed over ranks = 3 * 3 = 9 exactly;
    # reducing after the first micro-batch too would give 3 + 2 * 3 * ... != 9.
    assert res[0][1] == res[1][1] == [9.0] * 4
    # d/db per rank = 2 * (2 b)(rank + 1) = 8 (rank + 1), summed = 24
    assert res[0][2] == res[1][2] == [24.0] * 3
    # no all-reduce is in flight after the first micro-batch; two after the last
    assert res[0][3] == res[1][3] == [0, 2, 0, 2]
