"""Output-row band sharding on CPU with two gloo ranks: the bookkeeping of
RowBandMSETrainStep with the oracle standing in for the device kernels.

Each rank owns the output rows ``band(N, rank, 2)`` of the wide folded
config5s layer (footprints up to 768 sites on a 512-site chart, so many atoms
are halo atoms). It computes its Y band, dY band, G band = dY_band^T X (rows
outside the band zero), the banded atom gradient and its share of dX,
dY_band W_band; the gradient all-reduce (the halo exchange) and the dX
all-reduce must give the unsharded gradient and dX, the atoms whose partial
gradients are nonzero on both ranks must be the halo atoms ``meets_band``
names, and the optimizer step that follows must leave the atoms bitwise
identical on both ranks.
"""

import os
import socket

import numpy as np
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
        from torchcst_b200.shard import band, meets_band
        from torchcst_b200.train import dp_loss_scale
        out_axis, in_axis, spec = CASES["config5s"]
        d = load("config5s")
        p = d["p0"].astype(np.float32)
        n_out, n_in = out_axis.site_count, in_axis.site_count
        rows = 8
        rng = np.random.default_rng(11)
        x = rng.standard_normal((rows, n_in))
        t = rng.standard_normal((rows, n_out))
        lay = O.decode(out_axis, in_axis, spec, p)
        W = O.weight64(lay)
        r0, nb = band(n_out, rank, world)
        scale = dp_loss_scale(rows, n_out)
        dy_band = (x @ W[r0:r0 + nb].T - t[:, r0:r0 + nb]) * scale
        G = np.zeros((n_out, n_in))
        G[r0:r0 + nb] = dy_band.T @ x
        grad = torch.from_numpy(O.atom_gradients64(lay, G))
        partial = grad.clone()
        dx = torch.from_numpy(dy_band @ W[r0:r0 + nb])
        dist.all_reduce(grad)   # the halo exchange
        dist.all_reduce(dx)     # the dX shares
        full_dy = (x @ W.T - t) * (2.0 / (rows * n_out))
        full = O.atom_gradients64(lay, full_dy.T @ x)
        err_g = float(np.abs(grad.numpy() - full).max() / np.abs(full).max())
        err_x = float(np.abs(dx.numpy() - full_dy @ W).max() / np.abs(full_dy @ W).max())
        # Halo bookkeeping: nonzero partials exactly where the footprint meets the band.
        route = O.routing_table(lay)
        first = route["out_first_tile"] * 2 ** route["out_level"]
        length = route["out_count"] * 2 ** route["out_level"]
        meets = meets_band(first, length, n_out, r0, nb)
        nonzero = (partial.abs().sum(1) > 0).numpy()
        same_support = bool(np.array_equal(nonzero, meets))
        flags = torch.from_numpy(meets.astype(np.int64))
        dist.all_reduce(flags)
        halo = int((flags == world).sum())
        state = O.AdamState(0, np.zeros_like(p), np.zeros_like(p))
        new_p = O.optimizer_step(p, grad.numpy().astype(np.float32), state, spec, lr=1e-3)
        gathered = [torch.zeros(p.shape, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(np.ascontiguousarray(new_p, np.float32)))
        same = all(torch.equal(gathered[0], g) for g in gathered)
        if rank == 0:
            result.put((err_g, err_x, same_support, halo, same))
    finally:
        dist.destroy_process_group()


def test_two_rank_bands_sum_to_the_whole_step():
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, result)) for r in range(2)]
    for proc in procs:
        proc.start()
    try:
        err_g, err_x, same_support, halo, same = result.get(timeout=300)
    finally:
        for proc in procs:
            proc.join(timeout=60)
            if proc.is_alive():
                proc.kill()
    assert err_g < 1e-12 and err_x < 1e-12, (err_g, err_x)
    assert same_support
    assert halo > 0  # the wide layer has atoms on both bands
    assert same
    assert all(proc.exitcode == 0 for proc in procs)
