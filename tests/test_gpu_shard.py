"""Output-row band sharding on the GPU: one band equals the unsharded step, and
(with two or more GPUs) G bands over NCCL equal it too."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_single_band_matches_unsharded_step():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    sys.path.insert(0, HERE)
    from shard_worker import ROWS, build
    from torchcst_b200.shard import RowBandMSETrainStep
    from torchcst_b200.train import MSETrainStep
    dev = torch.device("cuda", 0)
    layer, opt, x, t = build(dev)
    step = RowBandMSETrainStep(layer, opt, ROWS)
    loss = float(step(x, t))
    ref_layer, ref_opt, _, _ = build(dev)
    ref = MSETrainStep(ref_layer, ref_opt, ROWS)
    ref_loss = float(ref(x, t))
    torch.cuda.synchronize()
    assert abs(loss - ref_loss) <= 1e-6 * abs(ref_loss)
    for c in range(4):
        a, b = step.grad[:, c], ref.grad[:, c]
        assert float((a - b).abs().max() / b.abs().max()) < 1e-4, c
    assert float((step.dx() - ref.dx).abs().max() / ref.dx.abs().max()) < 1e-4
    assert step.check_status() == 0


@pytest.mark.parametrize("world", [2])
def test_bands_over_nccl_match_unsharded_step(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", "29531", os.path.join(HERE, "shard_worker.py")]
    out = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-2000:]
