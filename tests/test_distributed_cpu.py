"""Host-side logic of the row-sharded path on CPU ranks (world size 2):
the communicator-id rendezvous, the shard bounds, and the sharded algebra of
one CG step (local row block of K·P, local partial dots, all-reduce) checked
against the unsharded float64 computation. The all-reduce stands in for NCCL
through torch.distributed's gloo backend (test-only)."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from mojogp_b200.distributed import exchange_id, shard_bounds


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rdv_worker(rank, world, port, q):
    payload = bytes(range(128)) if rank == 0 else None
    got = exchange_id(payload, rank, world, "127.0.0.1", port, timeout_s=60)
    q.put((rank, got))


@pytest.mark.parametrize("world", [2, 3])
def test_rendezvous_delivers_id_to_every_rank(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rdv_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=90) for _ in range(world))
    for p in procs:
        p.join(30)
        assert p.exitcode == 0
    assert all(v == bytes(range(128)) for v in res.values())


@pytest.mark.parametrize("n,world", [(10, 2), (1000, 3), (7, 8), (1_000_000, 8)])
def test_shard_bounds_partition(n, world):
    b = [shard_bounds(n, world, r) for r in range(world)]
    assert b[0][0] == 0 and b[-1][1] == n
    assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
    sizes = [r1 - r0 for r0, r1 in b]
    assert max(sizes) - min(sizes) <= 1


def _cg_step_worker(rank, world, port, q):
    import torch.distributed as dist
    from oracle import kernels as ok
    from mojogp_b200.kernel import RBF, make_ard_kernel
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    rng = np.random.default_rng(0)
    n, d, t = 300, 3, 5
    X = rng.standard_normal((n, d))
    Pm = rng.standard_normal((n, t))
    k = make_ard_kernel(RBF(ard=True), d)
    params = np.array([0.7, 1.1, 1.6, 1.3])
    r0, r1 = shard_bounds(n, world, rank)
    # local rows of (K + s I) P from replicated X and the full P
    Ap_local = ok.forward_matvec(k.to_spec(d), params, X, Pm, noise=0.1, rows=np.arange(r0, r1))
    pap_partial = np.sum(Pm[r0:r1] * Ap_local, axis=0)
    import torch
    tens = torch.from_numpy(pap_partial.copy())
    dist.all_reduce(tens)
    blocks = [torch.zeros((n // world + 1, t), dtype=torch.float64) for _ in range(world)]
    pad = torch.zeros((n // world + 1, t), dtype=torch.float64)
    pad[: r1 - r0] = torch.from_numpy(Ap_local)
    dist.all_gather(blocks, pad)
    full = np.concatenate([blocks[g].numpy()[: shard_bounds(n, world, g)[1] - shard_bounds(n, world, g)[0]]
                           for g in range(world)])
    q.put((rank, tens.numpy(), full))
    dist.destroy_process_group()


def test_sharded_cg_step_matches_unsharded():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cg_step_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(30)
        assert p.exitcode == 0
    from oracle import kernels as ok
    from mojogp_b200.kernel import RBF, make_ard_kernel
    rng = np.random.default_rng(0)
    n, d, t = 300, 3, 5
    X = rng.standard_normal((n, d))
    Pm = rng.standard_normal((n, t))
    k = make_ard_kernel(RBF(ard=True), d)
    Ap = ok.forward_matvec(k.to_spec(d), np.array([0.7, 1.1, 1.6, 1.3]), X, Pm, noise=0.1)
    for _, pap, full in res:
        np.testing.assert_allclose(pap, np.sum(Pm * Ap, axis=0), rtol=1e-12)
        np.testing.assert_allclose(full, Ap, rtol=1e-12)


class _GlooComm:
    """Stand-in for distributed.Communicator's host reductions over gloo (test-only)."""

    def __init__(self, rank, world):
        self.rank, self.world = rank, world

    def allreduce_sum(self, buf):
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(np.ascontiguousarray(buf, np.float64).copy())
        dist.all_reduce(t)
        return t.numpy()


class _RowwiseCache:
    """Stand-in for a prediction cache: mean / variance as fixed functions of each row."""

    rank = 8

    def predict(self, Xt, return_var=True):
        m = np.sin(Xt).sum(1).astype(np.float32)
        v = (1.0 + np.cos(Xt).sum(1) ** 2).astype(np.float32)
        return m, (v if return_var else None)


def _sharded_predict_worker(rank, world, port, m, q):
    import torch.distributed as dist
    from mojogp_b200.prediction import PredictionCache
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    Xt = np.random.default_rng(3).standard_normal((m, 3)).astype(np.float32)
    mean, var = PredictionCache.predict_sharded(_RowwiseCache(), Xt, _GlooComm(rank, world))
    q.put((rank, mean, var))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,m", [(2, 101), (3, 2), (2, 0)])
def test_sharded_prediction_assembles_every_row_on_every_rank(world, m):
    """X* sharding (PredictionCache.predict_sharded): each rank predicts its slice
    of the test rows, one all-reduce assembles all rows on every rank; ragged
    and empty slices included (m < world, m = 0)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_predict_worker, args=(r, world, port, m, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(30)
        assert p.exitcode == 0
    Xt = np.random.default_rng(3).standard_normal((m, 3)).astype(np.float32)
    ref_m, ref_v = _RowwiseCache().predict(Xt)
    for _, mean, var in res:
        assert mean.shape == (m,) and var.shape == (m,)
        np.testing.assert_array_equal(mean, ref_m)
        np.testing.assert_array_equal(var, ref_v)
