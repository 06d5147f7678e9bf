"""Data-parallel training through the native trainer and NCCL.

* Two ranks, each with half of the batch, must train like one rank with the
  whole batch (sums of per-rank gradients under the global loss normaliser),
  in the default sharded update form (reduce-scatter, Adam on each rank's
  shard, all-gather) and in the all-reduce form.
  The small exact-precision ReLU network: losses and parameters within 1e-5.
  The wide-MLP path at reduced width (four GELU layers, 3xTF32, He-normal; its
  layer-1 gradient all-reduced in row chunks and every bucket's Adam update on
  the communication stream): losses within 1e-4, parameters normwise within
  1e-4.  Needs 2 GPUs (skipped otherwise).
* A communicator whose peer never joins must end with JX_ETIMEOUT from the
  host watchdog, not hang (host-side failure; one GPU is enough).
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


SMALL = {"widths": [784, 256, 128, 10], "acts": ["relu", "relu"], "exact": True, "init": "xavier"}
WIDE = {"widths": [1024, 512, 512, 512, 512, 100], "acts": ["gelu"] * 4, "exact": False, "init": "he"}
WIDE_ALLREDUCE = dict(WIDE, sharded=False)


def _data(steps, batch, features=784, classes=10):
    rng = np.random.default_rng(7)
    xs = [rng.standard_normal((batch, features)).astype(np.float32) for _ in range(steps)]
    ys = [rng.integers(0, classes, batch).astype(np.float32) for _ in range(steps)]
    return xs, ys


def _init_params(net, init="xavier"):
    rng = np.random.default_rng(3)
    Ws, bs = [], []
    for l in range(len(net.widths) - 1):
        fi, fo = net.widths[l], net.widths[l + 1]
        if init == "he":
            Ws.append((rng.standard_normal((fi, fo)) * np.sqrt(2.0 / fi)).astype(np.float32))
        else:
            a = np.sqrt(6.0 / (fi + fo))
            Ws.append(rng.uniform(-a, a, (fi, fo)).astype(np.float32))
        bs.append(np.zeros(fo, np.float32))
    return net.pack(Ws, bs)


def _dp_worker(rank, world, port, steps, batch, out_dir, cfg=SMALL):
    import sys
    sys.path.insert(0, ROOT)
    import ctypes as C
    import datetime
    import importlib

    import torch
    import torch.distributed as dist
    jx = importlib.import_module("jax-rs_b200")
    torch.cuda.set_device(rank)
    jx.init(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    nid = jx.lib().jx_nccl_unique_id_size()
    idb = (C.c_char * nid)()
    if rank == 0:
        jx.call("jx_nccl_get_unique_id", idb)
    obj = [bytes(idb)]
    dist.broadcast_object_list(obj, src=0)
    idb = (C.c_char * nid).from_buffer_copy(obj[0])
    comm = C.c_void_p()
    jx.call("jx_nccl_init", idb, world, rank, 60000, C.byref(comm))
    per = batch // world
    prec = jx.PREC_EXACT if cfg["exact"] else jx.PREC_3XTF32
    net = jx.MLP(cfg["widths"], cfg["acts"], per, prec)
    net.set_params(_init_params(net, cfg["init"]))
    net.set_adam()
    net.attach_comm(comm, world, batch)
    if not cfg.get("sharded", True):
        jx.call("jx_mlp_set_dp_sharded", net.handle, 0)
    xs, ys = _data(steps, batch, cfg["widths"][0], cfg["widths"][-1])
    s = torch.cuda.current_stream().cuda_stream
    losses = []
    L = torch.empty(1, device="cuda")
    for x, y in zip(xs, ys):
        X = torch.from_numpy(x[rank * per:(rank + 1) * per].copy()).cuda()
        Y = torch.from_numpy(y[rank * per:(rank + 1) * per].copy()).cuda()
        net.step(X.data_ptr(), Y.data_ptr(), L.data_ptr(), s)
        torch.cuda.synchronize()
        losses.append(float(L.item()))
    params = net.get_params()
    np.save(os.path.join(out_dir, f"params{rank}.npy"), params)
    np.save(os.path.join(out_dir, f"loss{rank}.npy"), np.array(losses))
    del net
    jx.call("jx_nccl_destroy", comm)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("cfg,steps,batch", [(SMALL, 5, 128), (WIDE, 10, 256), (WIDE_ALLREDUCE, 10, 256)],
                         ids=["small_exact", "wide_gelu_3xtf32", "wide_allreduce_form"])
def test_two_rank_dp_matches_single_rank(jx, dev, tmp_path, cfg, steps, batch):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, steps, batch, str(tmp_path), cfg)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    # single rank, whole batch, in this process
    prec = jx.PREC_EXACT if cfg["exact"] else jx.PREC_3XTF32
    net = jx.MLP(cfg["widths"], cfg["acts"], batch, prec)
    net.set_params(_init_params(net, cfg["init"]))
    net.set_adam()
    xs, ys = _data(steps, batch, cfg["widths"][0], cfg["widths"][-1])
    L = dev.full((1,), np.nan)
    ref_losses = []
    for x, y in zip(xs, ys):
        X, Y = dev.put(x), dev.put(y)
        net.step(X.data_ptr(), Y.data_ptr(), L.data_ptr(), dev.stream)
        ref_losses.append(float(dev.get(L)[0]))
    ref = net.get_params()
    p0, p1 = np.load(tmp_path / "params0.npy"), np.load(tmp_path / "params1.npy")
    assert np.array_equal(p0, p1)  # ranks stay in lock-step
    l0, l1 = np.load(tmp_path / "loss0.npy"), np.load(tmp_path / "loss1.npy")
    if cfg["exact"]:
        assert np.abs(p0 - ref).max() <= 1e-5
        # each rank reports its half-batch loss under the global normaliser: they add up
        np.testing.assert_allclose(l0 + l1, ref_losses, atol=1e-5)
    else:
        d = np.linalg.norm((p0.astype(np.float64) - ref)) / np.linalg.norm(ref.astype(np.float64))
        assert d <= 1e-4, d
        assert np.abs((l0 + l1) - np.array(ref_losses)).max() <= 1e-4
        assert ref_losses[-1] < ref_losses[0]


def test_peer_that_never_joins_times_out(jx, dev):
    """Rank 0 of a 2-rank communicator whose rank 1 never starts: the host
    watchdog aborts the communicator and returns JX_ETIMEOUT."""
    import ctypes as C
    import time
    nid = jx.lib().jx_nccl_unique_id_size()
    idb = (C.c_char * nid)()
    jx.call("jx_nccl_get_unique_id", idb)
    comm = C.c_void_p()
    t0 = time.time()
    with pytest.raises(jx.JaxRsError) as e:
        jx.call("jx_nccl_init", idb, 2, 0, 3000, C.byref(comm))
    assert e.value.status == jx.JX_ETIMEOUT
    assert time.time() - t0 < 60
    assert not comm.value


def test_nccl_timeout_default_from_environment(jx, dev):
    """jx_nccl_init with timeout_ms = 0 takes JAXRS_NCCL_TIMEOUT_MS: a peer
    that never joins ends the call after about that long."""
    import ctypes as C
    import time
    nid = jx.lib().jx_nccl_unique_id_size()
    idb = (C.c_char * nid)()
    jx.call("jx_nccl_get_unique_id", idb)
    comm = C.c_void_p()
    os.environ["JAXRS_NCCL_TIMEOUT_MS"] = "2000"
    try:
        t0 = time.time()
        with pytest.raises(jx.JaxRsError) as e:
            jx.call("jx_nccl_init", idb, 2, 0, 0, C.byref(comm))
        assert e.value.status == jx.JX_ETIMEOUT
        assert "2000 ms" in e.value.message
        assert time.time() - t0 < 60
    finally:
        del os.environ["JAXRS_NCCL_TIMEOUT_MS"]
