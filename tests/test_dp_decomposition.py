"""CPU, world size 2 (gloo): the data-parallel decomposition the trainer uses.

Each rank holds half of the batch and computes the softmax-cross-entropy
adjoint with the *global* element count as normaliser; summing the ranks'
weight gradients (the all-reduce) must give the whole-batch gradient of the
reference's loss.  Computed with the oracle's C restatement.
"""
import os
import socket

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _grad(O, x, y, W, b, count):
    z = O.dense_fwd(x, W, b)
    p = O.softmax_rows(z)
    t = O.one_hot(y, W.shape[1])
    dz = O.softmax_xent_bwd(p, t) * np.float32(z.size / count)  # adjoint renormalised to `count`
    return O.matmul(O.transpose(x), dz.astype(np.float32)), O.col_sum(dz.astype(np.float32))


def _grad_gelu2(O, x, y, W1, b1, W2, b2, count):
    """Two-layer GELU network (the wide MLP's structure): dW1, dW2 under the
    loss normaliser `count`; backward dz1 = (dz2 W2^T) * gelu'(pre1)."""
    pre = O.dense_fwd(x, W1, b1)
    h = O.unary("gelu", pre)
    z = O.dense_fwd(h, W2, b2)
    p = O.softmax_rows(z)
    t = O.one_hot(y, W2.shape[1])
    dz2 = (O.softmax_xent_bwd(p, t) * np.float32(z.size / count)).astype(np.float32)
    gW2 = O.matmul(O.transpose(h), dz2)
    dz1 = (O.matmul(dz2, O.transpose(W2)) * O.gelu_grad(pre)).astype(np.float32)
    gW1 = O.matmul(O.transpose(x), dz1)
    return gW1, gW2


def _worker_gelu(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist

    import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(1)
    B, K, H, C = 64, 24, 32, 9
    x = rng.standard_normal((B, K)).astype(np.float32)
    y = rng.integers(0, C, B).astype(np.float32)
    W1 = (rng.standard_normal((K, H)) * np.sqrt(2.0 / K)).astype(np.float32)
    W2 = (rng.standard_normal((H, C)) * np.sqrt(2.0 / H)).astype(np.float32)
    b1, b2 = np.zeros(H, np.float32), np.zeros(C, np.float32)
    per = B // world
    sl = slice(rank * per, (rank + 1) * per)
    g1, g2 = _grad_gelu2(O, x[sl], y[sl], W1, b1, W2, b2, B * C)
    t1, t2 = torch.from_numpy(g1), torch.from_numpy(g2)
    dist.all_reduce(t1)
    dist.all_reduce(t2)
    if rank == 0:
        f1, f2 = _grad_gelu2(O, x, y, W1, b1, W2, b2, B * C)
        q.put((float(np.abs(t1.numpy() - f1).max()), float(np.abs(t2.numpy() - f2).max()),
               float(max(np.abs(f1).max(), np.abs(f2).max()))))
    dist.destroy_process_group()


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist

    import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(0)
    B, K, C = 64, 20, 7
    x = rng.standard_normal((B, K)).astype(np.float32)
    y = rng.integers(0, C, B).astype(np.float32)
    W = rng.standard_normal((K, C)).astype(np.float32)
    b = rng.standard_normal(C).astype(np.float32)
    per = B // world
    gW, gb = _grad(O, x[rank * per:(rank + 1) * per], y[rank * per:(rank + 1) * per], W, b, B * C)
    tW, tb = torch.from_numpy(gW), torch.from_numpy(gb)
    dist.all_reduce(tW)
    dist.all_reduce(tb)
    if rank == 0:
        fW, fb = _grad(O, x, y, W, b, B * C)
        q.put((float(np.abs(tW.numpy() - fW).max()), float(np.abs(tb.numpy() - fb).max()),
               float(np.abs(fW).max())))
    dist.destroy_process_group()


def _run(target):
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_allreduced_gelu_gradients_equal_full_batch_gradient(oracle):
    """The same decomposition through a GELU hidden layer (the wide MLP)."""
    d1, d2, scale = _run(_worker_gelu)
    assert d1 <= 1e-6 * max(1.0, scale) and d2 <= 1e-6 * max(1.0, scale)


def test_allreduced_half_batch_gradients_equal_full_batch_gradient(oracle):
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    dW, db, scale = res
    assert dW <= 1e-6 * max(1.0, scale) and db <= 1e-6 * max(1.0, scale)
