"""Token-sharded DiT stack across real GPUs (-m gpu; needs >= 2 GPUs).

Launches tests/mgpu_stack_check.py under torchrun (one process per GPU,
copy engines or NCCL for the data path, gloo only for bootstrap) and compares the gathered
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


@pytest.mark.parametrize("exchange", ["ce", "nccl"])
@pytest.mark.parametrize("overlap", ["0", "1"])
def test_sharded_stack_equals_single_gpu(gpu, ops, overlap, exchange):
    """overlap=0 with the attention's stream-K tail off: bit-identical to one
    GPU; overlap=1 (K/V exchange behind attention over the rank's own keys)
    with the default tail: within the bf16 aggregate bar, since both change
    the fp32 summation order.  The K/V rows of a split sample move either by
    copy-engine pushes into the peers' IPC-shared key buffers, ordered by
    sequence flags (exchange=ce, the default), or by the NCCL all-gather."""
    n = ops.get_device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = 4 if n >= 4 else 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SF_KV_OVERLAP=overlap, SF_KV_EXCHANGE=exchange)
    if overlap == "0":
        env["SF_ATTN_SPLIT"] = "0"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(29533 + int(overlap) + (2 if exchange == "nccl" else 0)), os.path.join(HERE, "mgpu_stack_check.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "[mgpu] OK" in r.stdout
