"""scaffolding_b200 -- a B200-native (sm_100a) matmul engine for Scaffolding.

Drop-in for the reference framework's matmul hot path: ``GpuTensor.matmul``,
the fused linear forward behind ``nn.Linear`` / ``F.linear``, the
strided-batched QK^T / PV products behind attention, and the M-sharded
multi-GPU path that replaces ``nn/parallel.py``'s host round-trips.

Modules:
  _cuda_ops   the reference ``_cuda_ops`` surface (GpuTensor, dev_*, cuda_*, runtime)
  nn          Linear / functional.linear / scaled_dot_product_attention on GpuTensors
  dit         DiT block linears used by the benchmark
  engine      thin wrappers over the C ABI (include/sf_engine.h)
  build       compiles libsf_engine.so (importable without the library)

Importing any module that touches the engine loads ``libsf_engine.so`` and
raises ``ImportError`` if it has not been built; there is no CPU fallback.
"""
__version__ = "0.1.0"

_LAZY = {"GpuTensor", "gputensor_from_numpy", "gputensor_to_numpy"}


def __getattr__(name):
    if name in _LAZY:
        from . import _cuda_ops
        return getattr(_cuda_ops, name)
    raise AttributeError(name)
