"""Fused MSE training step of one B200 CSTLinear (forward, backward, CSTAdamW).

Computes exactly what ``y = layer(x); ((y - t)**2).mean().backward();
optimizer.step()`` computes, without autograd bookkeeping: the MSE upstream
gradient is written over Y in one pass (with its loss partials and max |dY|),
every buffer is allocated once, and the step is a fixed sequence of native
launches on the current stream:

    decode/route -> bin sort (count, column prefix, scatter) | site values ->
    weight (mass cache, owner-pair coefficients and expansion, tile gather with
    max |W|, f16 split) | scalar fetch, f16 split of X -> GEMM Y -> MSE dY ->
    f16 split of dY -> GEMM dX | GEMM dW (split-K) -> pullback (split-K sum,
    four footprint classes, owner-pair projection and gradients, wide atoms) ->
    optimizer

The optimizer reads its per-step scalars (bias corrections) from a pinned host
ring through its device mapping (the host writes the step's slot before
enqueuing it), so :meth:`capture` can record the whole sequence as one CUDA
graph per input buffer pair and replay it with the host doing only the scalar
write, and no copy in front of the replay.

With ``process_group`` set (data parallel, rows sharded across ranks, atoms
replicated), the loss is scaled by the global row count and the atom gradient
is all-reduced (sum) before the optimizer, so every rank applies the identical
update. Captured steps then replay two graphs per step, the gradient and the
optimizer, with the all-reduce issued between them; neither graph holds a
collective.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N
from . import runtime as R
from .linear import CSTLinear
from .optim import CSTAdamW


def dp_loss_scale(rows: int, n_out: int, world_rows: int | None = None) -> float:
    """float32 dY scale of the mean-squared error over ``world_rows`` rows (all
    ranks) of ``n_out`` outputs; ``rows`` when there is no process group."""
    total = rows if world_rows is None else int(world_rows)
    return float(torch.tensor(2.0 / (total * n_out), dtype=torch.float32))


def dp_reduce_gradient(grad: torch.Tensor, process_group=None) -> torch.Tensor:
    """Sum the per-rank atom gradients in place (no-op without a group)."""
    if process_group is not None:
        torch.distributed.all_reduce(grad, group=process_group)
    return grad


class OptimizerScalars:
    """Device-side CSTAdamW step of one layer for captured or eager steps: the
    host computes the step's scalars (bias corrections) and writes them into a
    pinned ring that the fused optimizer kernel reads through its device
    mapping, so no host-to-device copy stands in front of a replay."""

    def __init__(self, layer: CSTLinear, optimizer: CSTAdamW, device):
        self.layer, self.opt = layer, optimizer
        self._ring = R.ScalarRing(device)
        self._state = None
        self._kind = None

    def _upload(self, h):
        """Write the next optimizer launch's scalars into the ring."""
        self._ring.write(h)

    def _advance(self):
        """Host side of one optimizer step: step count and scalars to the device.
        Returns False when the learning rate is 0 (the step leaves p unchanged)."""
        p = self.layer.atoms.p
        out = self.opt.site_step(p)
        p.grad = self.grad
        if out is None:
            return False
        h, self._state, self._kind = out
        self._upload(h)
        return True

    def check_status(self):
        """Read and clear the device status word once (a host synchronization;
        call it off the hot path, e.g. after a run of steps). Raises
        ``RuntimeError`` if any kernel since the last check flagged invalid
        atoms or gave up a bounded wait: the steps since then may hold partial
        results."""
        code = int(self.ws.status.item())
        if code:
            self.ws.status.zero_()
            raise RuntimeError(f"device status {code:#x}: {R.status_error(code)}")
        return 0

    def _fetch(self, stream):
        """Enqueue the device copy of this step's ring slot on ``stream``."""
        self._ring.fetch(self.ws.status, stream)

    def _launch_opt(self, fetched=False):
        """Enqueue the optimizer step; ``fetched``: the step's slot was already
        fetched earlier in the step (on a stream joined before this one)."""
        p = self.layer.atoms.p
        state = self._state
        stream = R._stream(p.device)
        if not fetched:
            self._fetch(stream)
        self._ring.launch(p, self.grad, state["exp_avg"], state["exp_avg_sq"], self._kind, stream)


class MSETrainStep(OptimizerScalars):
    LAUNCHES_PER_STEP = 27  # native kernels; torch adds the loss sum and one clear

    def __init__(self, layer: CSTLinear, optimizer: CSTAdamW, rows: int, *, need_dx=True,
                 process_group=None, world_rows=None):
        super().__init__(layer, optimizer, layer.atoms.p.device)
        self.rows = int(rows)
        self.need_dx = need_dx
        self.pg = process_group
        p = layer.atoms.p
        dev = p.device
        plan = layer._plan
        self.plan = plan
        self.ws = layer._workspace(dev)
        A = p.shape[0]
        self.atoms = A
        f32 = torch.float32
        self.table = torch.empty(max(plan.table_bytes(A) // 4, 1), dtype=f32, device=dev)
        self.scratch = self.ws.scratch(A)
        self.w = torch.empty(plan.n_out, plan.n_in, dtype=f32, device=dev)
        # absmax words (zeroed together each step) and scales of the W, X, dY splits
        self.amax = torch.zeros(3, dtype=f32, device=dev)
        self.scales = torch.ones(3, dtype=f32, device=dev)
        self.w16 = R.F16Split(plan.n_out, plan.n_in, dev, amax=self.amax[0:1],
                              scale=self.scales[0:1])
        self.x16 = R.F16Split(self.rows, plan.n_in, dev, amax=self.amax[1:2],
                              scale=self.scales[1:2])
        self.dy16 = R.F16Split(self.rows, plan.n_out, dev, amax=self.amax[2:3],
                               scale=self.scales[2:3])
        self.y = torch.empty(self.rows, plan.n_out, dtype=f32, device=dev)  # dY
        self.dx = torch.empty(self.rows, plan.n_in, dtype=f32, device=dev) if need_dx else None
        self.split = R.weight_split_k(plan, self.rows)
        self.ldg = R.pad4(plan.n_in)
        self.gstride = plan.n_out * self.ldg
        self.g = torch.empty(self.split * self.gstride, dtype=f32, device=dev)
        self.grad = torch.empty(A, 4, dtype=f32, device=dev)
        self.partial = torch.empty(1024, dtype=torch.float64, device=dev)  # loss partials
        self.scale = dp_loss_scale(self.rows, plan.n_out, world_rows)
        self.nblocks = ctypes.c_int32(0)
        self._graphs = {}
        self._opt_graph = None
        # Side stream for the branches that do not depend on the main chain
        # (X split during weight assembly; dX GEMM during dW GEMM + pullback).
        self._side = torch.cuda.Stream(dev)

    # -- pieces --------------------------------------------------------------------

    def _launch(self, x, target, optimize=True):
        """Enqueue the step's kernels (and the gradient all-reduce) on the current
        stream; returns the loss."""
        loss = self._launch_grad(x, target, fetch=optimize)
        dp_reduce_gradient(self.grad, self.pg)
        if optimize:
            self._launch_opt(fetched=True)
        return loss

    def _launch_grad(self, x, target, fetch=False):
        """Forward and backward kernels up to this rank's atom gradient; with
        ``fetch``, also this step's optimizer scalars (side stream, beside the
        decode)."""
        plan, ws, vp = self.plan, self.ws, R._vp
        p = self.layer.atoms.p
        main = torch.cuda.current_stream(p.device)
        side = self._side
        st, st2 = main.cuda_stream, side.cuda_stream
        oa, ia = ctypes.byref(plan.out_axis), ctypes.byref(plan.in_axis)
        lib = N.load()
        A, rows = self.atoms, self.rows
        w16, x16, dy16 = self.w16, self.x16, self.dy16

        def split(sp, src, ld, stream):
            N.check(lib.tcst_absmax(vp(src), sp.rows, sp.cols, ld, vp(sp.amax), stream), "absmax")
            N.check(lib.tcst_split_f16(vp(src), sp.rows, sp.cols, ld, vp(sp.amax), vp(sp.hi),
                                       vp(sp.lo), sp.ld, vp(sp.scale), stream), "split")

        def gemm(M, N_, K, a, a_mn, b, b_mn, c, ldc, split=1, sstride=0, what="gemm",
                 stream=st):
            N.check(lib.tcst_gemm_f16x3(M, N_, K, vp(a.hi), vp(a.lo), a.ld, a_mn, vp(a.scale),
                                        vp(b.hi), vp(b.lo), b.ld, b_mn, vp(b.scale), vp(c), ldc,
                                        split, sstride, vp(ws.status), stream), what)

        self.amax.zero_()
        side.wait_stream(main)  # X split runs beside decode and weight assembly
        if fetch:
            self._fetch(st2)
        split(x16, x, x.stride(0), st2)
        N.check(lib.tcst_decode_route(vp(p), A, oa, ia, ctypes.byref(plan.coords), vp(self.table),
                                      None, None, vp(ws.status), st), "decode")
        N.check(lib.tcst_assemble_weight_f16(vp(self.table), A, oa, ia, vp(self.scratch),
                                             self.scratch.numel() * 4, vp(self.w), plan.n_in,
                                             vp(w16.amax), vp(w16.hi), vp(w16.lo), w16.ld,
                                             vp(w16.scale), st), "weight")
        main.wait_stream(side)
        # Y, then dY in place with the loss partials and max |dY| (a separate
        # pass measured faster than folding the loss into the GEMM epilogue).
        gemm(rows, plan.n_out, plan.n_in, x16, 0, w16, 0, self.y, plan.n_out, what="gemm y")
        N.check(lib.tcst_mse_grad_f32(vp(self.y), vp(target), rows, plan.n_out, plan.n_out,
                                      ctypes.c_float(self.scale), vp(self.y), plan.n_out,
                                      vp(self.partial), ctypes.byref(self.nblocks),
                                      vp(dy16.amax), st), "mse")
        N.check(lib.tcst_split_f16(vp(self.y), rows, plan.n_out, plan.n_out, vp(dy16.amax),
                                   vp(dy16.hi), vp(dy16.lo), dy16.ld, vp(dy16.scale), st),
                "split dy")
        side.wait_stream(main)  # dX and the loss reduction beside dW and the pullback
        if self.need_dx:
            gemm(rows, plan.n_in, plan.n_out, dy16, 0, w16, 1, self.dx, plan.n_in, what="gemm dx",
                 stream=st2)
        with torch.cuda.stream(side):
            loss = self.partial[: self.nblocks.value].sum() / (rows * plan.n_out)
        if not torch.cuda.is_current_stream_capturing():
            loss.record_stream(main)  # made on the side stream, read on the main one
        gemm(plan.n_out, plan.n_in, rows, dy16, 1, x16, 1, self.g, self.ldg, self.split,
             self.gstride, what="gemm dw")
        N.check(lib.tcst_pullback(vp(self.table), A, oa, ia, vp(self.g), self.ldg, self.split,
                                  self.gstride, vp(self.grad), st), "pullback")
        main.wait_stream(side)
        return loss

    # -- public --------------------------------------------------------------------

    def __call__(self, x, target):
        """Run one step on device tensors x [rows, in], target [rows, out]; returns the
        loss as a 0-d float64 device tensor (no host synchronization)."""
        with R.on_device(self.layer.atoms.p.device):
            return self._step(x, target)

    def _step(self, x, target):
        optimize = self._advance()
        key = (x.data_ptr(), target.data_ptr())
        graph = self._graphs.get(key) if optimize else None
        if graph is not None:
            graph[0].replay()
            if self.pg is not None:
                dp_reduce_gradient(self.grad, self.pg)
                self._opt_graph.replay()
            return graph[1]
        return self._launch(x, target, optimize)

    def capture(self, pairs):
        """Record one CUDA graph per (x, target) buffer pair; later calls with those
        buffers replay it. Needs one eager step first (one-time kernel setup). With
        a process group the optimizer is a second graph and the all-reduce runs
        between the two."""
        if self._state is None:
            raise RuntimeError("run one eager step before capturing")
        with R.on_device(self.layer.atoms.p.device):
            self._capture(pairs)

    def _capture(self, pairs):
        torch.cuda.synchronize()
        for x, target in pairs:
            key = (x.data_ptr(), target.data_ptr())
            if key in self._graphs:
                continue
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                loss = self._launch_grad(x, target, fetch=True)
                if self.pg is None:
                    self._launch_opt(fetched=True)
            self._graphs[key] = (graph, loss)
        if self.pg is not None and self._opt_graph is None:
            self._opt_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self._opt_graph):
                self._launch_opt(fetched=True)
        torch.cuda.synchronize()

    def release(self):
        """Drop the captured graphs."""
        self._graphs.clear()
        self._opt_graph = None


class GraphedStep:
    """One CUDA graph per input-buffer set for a training step written with the
    drop-in API::

        def step(x, target):
            optimizer.zero_grad(set_to_none=True)
            loss = loss_fn(model(x), target)
            loss.backward()
            optimizer.step()
            return loss

        graphed = GraphedStep(step, optimizer)
        loss = graphed(x, target)   # every call is exactly one training step

    The first ``warmup`` calls run eagerly on a side stream (the warm-up CUDA
    graph capture needs); the next call with a given set of input buffers
    captures the step and every later call with those buffers replays it, the
    host doing only the optimizer's per-step scalar refresh
    (:meth:`CSTAdamW.refresh_captured`). Inputs are identified by their device
    pointers: pass the same buffers (refilled) to reuse a graph. Returns the
    step function's result; for replays it is the captured output tensor,
    overwritten by the next replay. Ordinary parameters need a capturable
    optimizer group (``capturable=True``); CSTLinear status checks run on the
    device inside replays (read them with ``check_status``)."""

    def __init__(self, step_fn, optimizer: CSTAdamW, *, warmup: int = 3):
        if int(warmup) < 1:
            raise ValueError("GraphedStep needs at least one eager warm-up step")
        self.step_fn, self.opt, self.warmup = step_fn, optimizer, int(warmup)
        self._eager = 0
        self._graphs = {}
        self._side = None

    def __call__(self, *tensors):
        key = tuple(t.data_ptr() for t in tensors)
        entry = self._graphs.get(key)
        if entry is None and self._eager < self.warmup:
            self._eager += 1
            main = torch.cuda.current_stream()
            if self._side is None:
                self._side = torch.cuda.Stream(main.device)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                out = self.step_fn(*tensors)
            main.wait_stream(self._side)
            return out
        if entry is None:
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = self.step_fn(*tensors)
            entry = self._graphs[key] = (graph, out)
        self.opt.refresh_captured()
        entry[0].replay()
        return entry[1]

    def release(self):
        """Drop the captured graphs (and their memory pools)."""
        self._graphs.clear()

