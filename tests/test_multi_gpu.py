"""Token-sharded DiT stack across real GPUs (-m gpu; needs >= 2 GPUs).

Launches tests/mgpu_stack_check.py under torchrun (one process per GPU,
NCCL for the data path, gloo only for bootstrap) and compares the gathered
sharded output with the single-GPU output: bit for bit on the path whose
fp32 summation order does not depend on the sharding, else within the bf16
aggregate bar.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("overlap", ["0", "1"])
def test_sharded_stack_equals_single_gpu(gpu, ops, overlap):
    """overlap=0 with the attention's split dispatch off: bit-identical to
    one GPU; overlap=1 (K/V all-gather on a side stream behind attention over
    the rank's own keys) with the default split dispatch: within the bf16
    aggregate bar, since both change the fp32 summation order."""
    n = ops.get_device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = 4 if n >= 4 else 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SF_KV_OVERLAP=overlap)
    if overlap == "0":
        env["SF_ATTN_SPLIT"] = "0"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(29533 + int(overlap)), os.path.join(HERE, "mgpu_stack_check.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "[mgpu] OK" in r.stdout
