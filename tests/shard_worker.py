"""One rank of the row-band sharding check (run by tests/test_gpu_shard.py under
torchrun): three sharded MSE steps against the single-GPU steps on rank 0
(loss, atom gradient, dX and atoms within 1e-4), with the atoms and Adam
moments identical on every rank after each step."""

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from torchcst_b200 import CSTAdamW, CSTLinear, ChebyshevSpec, chart_presets, kernels  # noqa: E402
from torchcst_b200.shard import RowBandMSETrainStep  # noqa: E402
from torchcst_b200.train import MSETrainStep  # noqa: E402

N_SITES, ATOMS, ROWS = 512, 4096, 256


def build(device):
    torch.manual_seed(0)
    grid = chart_presets.regular_grid(N_SITES, geometry="flat_torus")
    kernel = kernels.product(kernels.cell_mass(ChebyshevSpec(modes=8)),
                             coordinates=kernels.rational_radius(radius_max=128.0))
    g = torch.Generator().manual_seed(1)
    p = torch.stack([torch.randn(ATOMS, generator=g) * 0.1, torch.rand(ATOMS, generator=g),
                     torch.rand(ATOMS, generator=g) * N_SITES,
                     torch.rand(ATOMS, generator=g) * N_SITES], 1)
    layer = CSTLinear(charts=(grid, grid), atoms=p, kernel=kernel, device=device, validate="off")
    opt = CSTAdamW(layer.parameters(), model=layer, lr=1e-3)
    x = torch.randn(ROWS, N_SITES, generator=g).to(device)
    t = torch.randn(ROWS, N_SITES, generator=g).to(device)
    return layer, opt, x, t


def main():
    dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    layer, opt, x, t = build(dev)
    step = RowBandMSETrainStep(layer, opt, ROWS, process_group=dist.group.WORLD)
    ok = torch.ones(1, device=dev)
    rel = lambda a, b: float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))
    if rank == 0:
        ref_layer, ref_opt, _, _ = build(dev)
        ref = MSETrainStep(ref_layer, ref_opt, ROWS)
    for k in range(3):
        loss = float(step(x, t))
        torch.cuda.synchronize()
        if step.check_status() != 0:
            ok.zero_()
        # Atoms and moments stay identical on every rank.
        st = opt.state[layer.atoms.p]
        for tensor in (layer.atoms.p.detach(), st["exp_avg"], st["exp_avg_sq"]):
            gathered = [torch.empty_like(tensor) for _ in range(world)]
            dist.all_gather(gathered, tensor.contiguous())
            if not all(torch.equal(gathered[0], g) for g in gathered):
                ok.zero_()
        if rank == 0:
            ref_loss = float(ref(x, t))
            torch.cuda.synchronize()
            errs = [rel(step.grad[:, c], ref.grad[:, c]) for c in range(4)]
            errs.append(rel(step.dx(), ref.dx))
            errs.append(rel(layer.atoms.p.detach(), ref_layer.atoms.p.detach()))
            print("step", k, "loss", loss, ref_loss, "errors", errs, flush=True)
            if abs(loss - ref_loss) > 1e-6 * abs(ref_loss) or max(errs) > 1e-4:
                ok.zero_()
    dist.broadcast(ok, 0)
    dist.destroy_process_group()
    sys.exit(0 if float(ok) == 1.0 else 1)


if __name__ == "__main__":
    main()
