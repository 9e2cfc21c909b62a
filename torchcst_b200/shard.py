"""One CSTLinear MSE training step sharded by output-row bands (one process per GPU).

Rank g of G owns output rows [r0, r0 + nb) with nb = N_out / G (a multiple of
32). Atoms, their AdamW moments, X and the target are replicated; every rank
decodes and sorts all atoms (O(A) work, small beside the band's work at the
sizes that shard). One step:

    W[r0:r0+nb, :] (window assembly, f16 split) | f16 split of X
    Y band = X W_band^T, then dY band = (Y band - T[:, band]) 2/(B N_out) with
      its loss partials and max |dY| (the band's own split scale)
    dW band = dY_band^T X and the banded pullback: each atom's gradient from
      the band's rows; atoms whose footprints cross band edges (the halo) get
      partial sums on several ranks
    | beside them: the band's share of dX, dY_band W_band (B x N_in, K = nb),
      all-reduced (sum) over the ranks on a second communicator, so every rank
      ends with the whole dX = sum over bands of dY_band W_band
    atom gradients: all-reduce (sum) -- the halo exchange (atoms inside one
      band add zeros elsewhere)
    CSTAdamW on every rank (identical)

NCCL carries the dX partial all-reduce (a reduce-scatter of the dX column
blocks and their all-gather), the halo-atom gradient reduction (the whole
[A, 4] gradient: 16 B per atom) and the loss sum. Work per rank is 1/G of the
weight assembly, of the three GEMMs and of the pullback (plus the halo).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as N
from . import runtime as R
from .linear import CSTLinear
from .optim import CSTAdamW
from .train import OptimizerScalars, dp_loss_scale


def band(n: int, rank: int, world: int):
    """(start, length) of rank's band of n sites: equal bands, 32-site aligned."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank out of range")
    if n % world or (n // world) % 32:
        raise ValueError(f"{n} sites do not split into {world} bands of a multiple of 32 sites")
    nb = n // world
    return rank * nb, nb


def meets_band(first, length, n: int, r0: int, nb: int):
    """Which cyclic footprints [first, first + length) (mod n) meet the band
    [r0, r0 + nb): elementwise over array-likes of first sites and lengths (the
    rule the banded pullback applies on the device). Atoms that meet several
    bands are the halo: their gradients are partial sums on each of them."""
    import numpy as np
    first = np.mod(np.asarray(first, np.int64), n)
    length = np.asarray(length, np.int64)
    if nb >= n:
        return length > 0
    end = first + length
    inside = (first < r0 + nb) & (r0 < end)          # no wrap past n
    wrapped = (end > n) & (r0 < end - n)              # the part past n, from site 0
    return (length > 0) & ((length >= n) | inside | wrapped)


class RowBandMSETrainStep(OptimizerScalars):
    """Eager MSE training step of one layer sharded by output-row bands over a
    process group (NCCL); ``process_group=None`` runs the whole layer as one band."""

    LAUNCHES_PER_STEP = 26  # native kernels (decode, site values, sort, window assembly, splits, GEMMs, banded pullback, scalar fetch, optimizer)

    def __init__(self, layer: CSTLinear, optimizer: CSTAdamW, rows: int, *, need_dx=True,
                 process_group=None):
        p = layer.atoms.p
        super().__init__(layer, optimizer, p.device)
        self.rows, self.need_dx, self.pg = int(rows), need_dx, process_group
        self.world = dist.get_world_size(process_group) if process_group is not None else 1
        self.rank = dist.get_rank(process_group) if process_group is not None else 0
        # A second communicator for the dX all-reduce, so that it runs beside
        # the dW GEMM, the pullback and the gradient all-reduce.
        self.pg_dx = (dist.new_group(dist.get_process_group_ranks(process_group))
                      if process_group is not None and need_dx else None)
        dev = p.device
        plan = layer._plan
        self.plan = plan
        self.ws = layer._workspace(dev)
        A = self.atoms = p.shape[0]
        B, no, ni = self.rows, plan.n_out, plan.n_in
        self.r0, self.nb = band(no, self.rank, self.world)
        f32 = torch.float32
        self.table = torch.empty(max(plan.table_bytes(A) // 4, 1), dtype=f32, device=dev)
        self.scratch = self.ws.scratch(A)
        # absmax words and scales: W band, X, dY band
        self.amax = torch.zeros(3, dtype=f32, device=dev)
        self.scales = torch.ones(3, dtype=f32, device=dev)
        self.w_band = torch.empty(self.nb, ni, dtype=f32, device=dev)
        self.w16b = R.F16Split(self.nb, ni, dev, amax=self.amax[0:1], scale=self.scales[0:1])
        self.x16 = R.F16Split(B, ni, dev, amax=self.amax[1:2], scale=self.scales[1:2])
        self.dy16 = R.F16Split(B, self.nb, dev, amax=self.amax[2:3], scale=self.scales[2:3])
        self.dx_full = torch.empty(B, ni, dtype=f32, device=dev) if need_dx else None
        self.y = torch.empty(B, no, dtype=f32, device=dev)  # Y band at columns [r0, r0 + nb)
        self.dy_band = torch.empty(B, self.nb, dtype=f32, device=dev)
        tiles = -(-self.nb // 128) * -(-ni // 256)
        self.split = int(max(1, min(8, -(-B // 32), 148 // max(tiles, 1))))
        self.ldg = R.pad4(ni)
        self.gstride = self.nb * self.ldg
        self.g = torch.empty(self.split * self.gstride, dtype=f32, device=dev)
        self.grad = torch.empty(A, 4, dtype=f32, device=dev)
        self.partial = torch.empty(1024, dtype=torch.float64, device=dev)
        self.loss_sum = torch.zeros(1, dtype=torch.float64, device=dev)
        self.scale = dp_loss_scale(B, no)
        self.nblocks = ctypes.c_int32(0)
        self._side = torch.cuda.Stream(dev)
        self._dx_side = torch.cuda.Stream(dev)
        self.marks = None  # a list: CUDA events at the phase boundaries of the next steps

    def _mark(self, name):
        if self.marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.marks.append((name, ev))

    def _gemm(self, M, N_, K, a_hi, a_lo, lda, a_mn, a_scale, b_hi, b_lo, ldb, b_mn, b_scale, c,
              ldc, split=1, sstride=0, stream=None, what="gemm"):
        st = stream if stream is not None else R._stream(self.layer.atoms.p.device)
        P = ctypes.c_void_p
        N.check(N.load().tcst_gemm_f16x3(M, N_, K, P(a_hi), P(a_lo), lda, a_mn, P(a_scale),
                                         P(b_hi), P(b_lo), ldb, b_mn, P(b_scale), P(c), ldc,
                                         split, sstride, R._vp(self.ws.status), st), what)

    def _launch_grad(self, x, target):
        plan, vp, lib = self.plan, R._vp, N.load()
        p = self.layer.atoms.p
        main = torch.cuda.current_stream(p.device)
        side = self._side
        st, st2 = main.cuda_stream, side.cuda_stream
        oa, ia = ctypes.byref(plan.out_axis), ctypes.byref(plan.in_axis)
        A, B, no, ni = self.atoms, self.rows, plan.n_out, plan.n_in
        r0, nb = self.r0, self.nb
        x16, dy16, w16b = self.x16, self.dy16, self.w16b
        pg = self.pg
        self._mark("start")
        self.amax.zero_()
        side.wait_stream(main)  # X split beside decode and weight assembly
        N.check(lib.tcst_absmax(vp(x), B, ni, x.stride(0), vp(x16.amax), st2), "absmax x")
        N.check(lib.tcst_split_f16(vp(x), B, ni, x.stride(0), vp(x16.amax), vp(x16.hi),
                                   vp(x16.lo), x16.ld, vp(x16.scale), st2), "split x")
        N.check(lib.tcst_decode_route(vp(p), A, oa, ia, ctypes.byref(plan.coords),
                                      vp(self.table), None, None, vp(self.ws.status), st),
                "decode")
        sb = self.scratch.numel() * 4
        N.check(lib.tcst_assemble_weight_window_f16(
            vp(self.table), A, oa, ia, vp(self.scratch), sb, r0, nb, 0, ni, vp(self.w_band), ni,
            vp(w16b.amax), vp(w16b.hi), vp(w16b.lo), w16b.ld, vp(w16b.scale), st), "weight band")
        main.wait_stream(side)
        self._mark("decode+sort+weights")
        y_band = self.y[:, r0:]
        self._gemm(B, nb, ni, x16.hi.data_ptr(), x16.lo.data_ptr(), x16.ld, 0,
                   x16.scale.data_ptr(), w16b.hi.data_ptr(), w16b.lo.data_ptr(), w16b.ld, 0,
                   w16b.scale.data_ptr(), y_band.data_ptr(), no, what="gemm y")
        N.check(lib.tcst_mse_grad_f32(vp(y_band), vp(target[:, r0:]), B, nb, no,
                                      ctypes.c_float(self.scale), vp(self.dy_band), nb,
                                      vp(self.partial), ctypes.byref(self.nblocks),
                                      vp(dy16.amax), st), "mse")
        torch.sum(self.partial[: self.nblocks.value], dim=0, keepdim=True, out=self.loss_sum)
        N.check(lib.tcst_split_f16(vp(self.dy_band), B, nb, nb, vp(dy16.amax), vp(dy16.hi),
                                   vp(dy16.lo), dy16.ld, vp(dy16.scale), st), "split dy")
        self._mark("gemm Y+loss+split")
        reduce_dx = None
        if self.need_dx:
            # The band's share of dX = dY_band W_band beside the dW GEMM and the
            # pullback, then its all-reduce on the second communicator.
            dxs = self._dx_side
            dxs.wait_stream(main)
            self._gemm(B, ni, nb, dy16.hi.data_ptr(), dy16.lo.data_ptr(), dy16.ld, 0,
                       dy16.scale.data_ptr(), w16b.hi.data_ptr(), w16b.lo.data_ptr(), w16b.ld, 1,
                       w16b.scale.data_ptr(), self.dx_full.data_ptr(), ni,
                       stream=dxs.cuda_stream, what="gemm dx")
            if self.pg_dx is not None:
                with torch.cuda.stream(dxs):
                    reduce_dx = dist.all_reduce(self.dx_full, group=self.pg_dx, async_op=True)
        self._gemm(nb, ni, B, dy16.hi.data_ptr(), dy16.lo.data_ptr(), dy16.ld, 1,
                   dy16.scale.data_ptr(), x16.hi.data_ptr(), x16.lo.data_ptr(), x16.ld, 1,
                   x16.scale.data_ptr(), self.g.data_ptr(), self.ldg, self.split, self.gstride,
                   what="gemm dw")
        N.check(lib.tcst_pullback_band(vp(self.table), A, oa, ia, vp(self.g), self.ldg,
                                       self.split, self.gstride, r0, nb, vp(self.grad), st),
                "pullback")
        self._mark("gemm dW+pullback")
        if pg is not None:
            dist.all_reduce(self.grad, group=pg)  # the halo exchange
            dist.all_reduce(self.loss_sum, group=pg)
        self._mark("gradient all-reduce")
        if self.need_dx:
            if reduce_dx is not None:
                reduce_dx.wait()
            main.wait_stream(self._dx_side)
            self._mark("dX all-reduce wait")
        return self.loss_sum[0] / (B * no)

    def __call__(self, x, target):
        """One step on this rank's device tensors x [rows, N_in] and target
        [rows, N_out] (replicated across ranks); returns the loss (0-d float64
        device tensor, identical on every rank)."""
        with R.on_device(self.layer.atoms.p.device):
            optimize = self._advance()
            loss = self._launch_grad(x, target)
            if optimize:
                self._launch_opt()
            self._mark("optimizer")
        return loss

    def dx(self):
        """dX [rows, N_in] of the last step (the sum of every band's share)."""
        if not self.need_dx:
            raise RuntimeError("built with need_dx=False")
        return self.dx_full
