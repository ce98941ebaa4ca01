"""scaffolding_b200 -- a B200-native (sm_100a) matmul engine for Scaffolding.

Drop-in for the reference framework's matmul hot path: ``GpuTensor.matmul``,
the fused linear forward behind ``nn.Linear`` / ``F.linear``, the
strided-batched QK^T / PV products behind attention, and the M-sharded
multi-GPU path that replaces ``nn/parallel.py``'s host round-trips.

Modules:
  _cuda_ops   the reference ``_cuda_ops`` surface (GpuTensor, dev_*, cuda_*, runtime)
  nn          Linear / functional.linear / scaled_dot_product_attention on GpuTensors
  parallel    token (M) sharding over one process per GPU + NCCL all-gather
  dit         DiT block linears and the 30-layer DiT stack used by the benchmark
  engine      thin wrappers over the C ABI (include/sf_engine.h)
"""
from . import _cuda_ops  # noqa: F401  (loads libsf_engine.so; raises if it is missing)
from ._cuda_ops import GpuTensor, gputensor_from_numpy, gputensor_to_numpy  # noqa: F401

__version__ = "0.1.0"
