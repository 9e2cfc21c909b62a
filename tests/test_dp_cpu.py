"""Data-parallel step semantics on CPU with two gloo ranks.

Each rank holds half of the rows and the full (replicated) atom table. It scales
dY by the global row count (``dp_loss_scale``), forms its share of G = dY^T X,
pulls back its atom gradient (the oracle stands in for the device kernels) and
sums the shares with ``dp_reduce_gradient``. The summed gradient must equal the
full-batch gradient, and the optimizer step that follows must leave the atoms
bitwise identical on both ranks.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import cst_oracle as O
from tests.golden_cases import CASES, load


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from torchcst_b200.train import dp_loss_scale, dp_reduce_gradient
        out_axis, in_axis, spec = CASES["config1"]
        d = load("config1")
        p = d["p0"].astype(np.float32)
        rng = np.random.default_rng(7)
        rows = 8
        x = rng.standard_normal((rows, in_axis.site_count)).astype(np.float32)
        t = rng.standard_normal((rows, out_axis.site_count)).astype(np.float32)
        lay = O.decode(out_axis, in_axis, spec, p)
        W = O.weight64(lay)
        share = slice(rank * rows // world, (rank + 1) * rows // world)
        xs, ts = x[share].astype(np.float64), t[share].astype(np.float64)
        scale = dp_loss_scale(rows // world, out_axis.site_count, rows)
        dy = (xs @ W.T - ts) * scale
        grad = torch.from_numpy(O.atom_gradients64(lay, dy.T @ xs).astype(np.float32))
        dp_reduce_gradient(grad, dist.group.WORLD)
        full_dy = (x.astype(np.float64) @ W.T - t) * (2.0 / (rows * out_axis.site_count))
        full = O.atom_gradients64(lay, full_dy.T @ x.astype(np.float64))
        err = float(np.abs(grad.numpy() - full).max() / np.abs(full).max())
        state = O.AdamState(0, np.zeros_like(p), np.zeros_like(p))
        new_p = O.optimizer_step(p, grad.numpy(), state, spec, lr=1e-3)
        gathered = [torch.zeros(p.shape, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(np.ascontiguousarray(new_p, np.float32)))
        same = all(torch.equal(gathered[0], g) for g in gathered)
        if rank == 0:
            result.put((err, same))
    finally:
        dist.destroy_process_group()


def test_two_rank_gradient_sum_and_identical_update():
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, result)) for r in range(2)]
    for proc in procs:
        proc.start()
    try:
        err, same = result.get(timeout=180)
    finally:
        for proc in procs:
            proc.join(timeout=60)
            if proc.is_alive():
                proc.kill()
    assert err < 1e-6
    assert same
    assert all(proc.exitcode == 0 for proc in procs)
