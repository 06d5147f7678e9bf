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
