"""MLP training restated with the oracle's C routines -- TEST INFRASTRUCTURE ONLY.

The reference trains its MLP example (examples/mlp_training.rs:19-36,94-145)
with finite differences and SGD; the 784-256-128-10 training workload runs Adam.
This module composes the reference's own pieces in the order a jax-rs program
would: Array::matmul (src/ops/linalg.rs:215-232), broadcast bias add
(src/ops/manipulation.rs:919-946), nn::relu (src/nn.rs:22-26), per-row
nn::softmax (:155-168), nn::one_hot (:205-221), nn::cross_entropy_loss
(:300-318) and optim::adam_update (src/optim.rs:138-189).  The backward pass
is the analytic derivative of that forward (the reference's grad cannot see
through these untraced functions):
  dL/dlogits = softmax-xent adjoint (epsilon kept),
  dW = h_prev^T dz, db = column sums of dz, dh = dz W^T, dz = dh * (pre > 0).

Inputs follow the configuration "regenerated per step from seed 0": step s
uses keys = PRNGKey::from_seed(0).split_n(steps); (kx, ky) = keys[s].split();
x = normal(kx), labels = randint(ky, 0, classes).  Seeding each step through
split_n avoids from_seed(0)'s all-zero xorshift state (src/random.rs:29-32).
"""
from __future__ import annotations

import numpy as np

from . import (adam_update, col_sum, cross_entropy, dense_fwd, gelu_grad, key_from_seed, matmul, normal, one_hot,
               randint, softmax_rows, softmax_xent_bwd, transpose, unary, uniform_range)


def xavier_params(widths, seed=1):
    """Xavier-uniform weights, a = sqrt(6/(fan_in+fan_out)), from
    uniform_range (src/random.rs:161-181) with keys from_seed(seed).split_n(L);
    zero biases."""
    keys = key_from_seed(seed).split_n(len(widths) - 1)
    Ws, bs = [], []
    for l in range(len(widths) - 1):
        fi, fo = widths[l], widths[l + 1]
        a = float(np.float32(np.sqrt(6.0 / (fi + fo))))
        Ws.append(uniform_range(keys[l], fi * fo, -a, a).reshape(fi, fo))
        bs.append(np.zeros(fo, np.float32))
    return Ws, bs


def batches(steps, batch, features, classes, seed=0):
    keys = key_from_seed(seed).split_n(steps)
    out = []
    for s in range(steps):
        kx, ky = keys[s].split()
        x = normal(kx, batch * features).reshape(batch, features)
        y = randint(ky, batch, 0, classes)
        out.append((x, y))
    return out


def _act(name, z):
    if name == "relu":
        return np.maximum(z, np.float32(0.0))  # nn::relu (f32::max)
    if name == "gelu":
        return unary("gelu", z)  # nn::gelu, src/nn.rs:111-122
    return z


def _act_grad(name, pre):
    if name == "relu":
        return (pre > 0).astype(np.float32)
    if name == "gelu":
        return gelu_grad(pre)
    return np.ones_like(pre)


def train(Ws, bs, data, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, nthreads=8, acts=None):
    """Runs len(data) Adam steps; returns (losses, Ws, bs).  acts names each
    hidden layer's activation ("relu", the default, or "gelu"); with gelu the
    backward multiplies by its derivative (dz = dh * gelu'(pre))."""
    Ws = [w.copy() for w in Ws]
    bs = [b.copy() for b in bs]
    L = len(Ws)
    acts = list(acts) if acts is not None else ["relu"] * (L - 1)
    mW = [np.zeros_like(w) for w in Ws]
    vW = [np.zeros_like(w) for w in Ws]
    mb = [np.zeros_like(b) for b in bs]
    vb = [np.zeros_like(b) for b in bs]
    losses = []
    for step, (x, y) in enumerate(data, start=1):
        hs, pres = [x], []
        h = x
        for l in range(L):
            z = dense_fwd(h, Ws[l], bs[l], nthreads)
            if l < L - 1:
                pres.append(z)
                h = _act(acts[l], z)
            else:
                h = z
            hs.append(h)
        p = softmax_rows(hs[-1])
        t = one_hot(y, Ws[-1].shape[1])
        losses.append(float(cross_entropy(p, t)))
        dz = softmax_xent_bwd(p, t)
        for l in range(L - 1, -1, -1):
            gW = matmul(transpose(hs[l]), dz, nthreads)
            gb = col_sum(dz)
            if l > 0:
                dh = matmul(dz, transpose(Ws[l]), nthreads)
                dz = (dh * _act_grad(acts[l - 1], pres[l - 1])).astype(np.float32)
            Ws[l], mW[l], vW[l] = adam_update(Ws[l], gW, mW[l], vW[l], lr, b1, b2, eps, step, step == 1)
            bs[l], mb[l], vb[l] = adam_update(bs[l], gb, mb[l], vb[l], lr, b1, b2, eps, step, step == 1)
    return losses, Ws, bs
