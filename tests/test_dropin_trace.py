"""The calls the reference's own Python makes into ``_cuda_ops`` (recorded by
``tests/golden/make_dropin_trace.py`` from the reference's nn.Linear, F.silu,
F.softmax, sf.matmul / matmul_nt and F.scaled_dot_product_attention on cuda
tensors), replayed through the drop-in module.

* CPU: every function the reference called is provided by
  ``scaffolding_b200._cuda_ops`` (not one of its out-of-scope stubs), with a
  signature that accepts the recorded arguments.
* GPU (-m gpu): the calls run in recorded order, each taking the drop-in's own
  results of the earlier calls, and every result matches the recorded one:
  uploads bit for bit, computed results within the 1e-5 relative Frobenius
  bar.
"""
import inspect
import json
import os

import numpy as np
import pytest

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TRACE = json.load(open(os.path.join(HERE, "dropin_trace.json")))["calls"]
# uploads and device moves copy bytes; everything else (downloads of computed
# results included) is checked against the fp32 bar
EXACT = {"gputensor_from_numpy", "gputensor_to_device", "set_device"}


def _arrays():
    return np.load(os.path.join(HERE, "dropin_arrays.npz"))


def test_reference_calls_are_provided(ops):
    names = sorted({c["fn"] for c in TRACE})
    assert {"dev_linear_forward", "cuda_linear_forward", "dev_batched_matmul_nt",
            "dev_softmax", "cuda_silu"} <= set(names)
    for name in names:
        fn = getattr(ops, name)
        assert name not in ops._OUT_OF_SCOPE, name
        n_args = max(len(c["args"]) for c in TRACE if c["fn"] == name)
        inspect.signature(fn).bind(*([None] * n_args))


@pytest.mark.gpu
def test_replay_reference_calls(gpu, ops):
    from oracle import oracle as O
    arr = _arrays()
    live = {}
    for i, call in enumerate(TRACE):
        args = []
        for a in call["args"]:
            if isinstance(a, dict) and "tensor" in a:
                args.append(live[a["tensor"]])
            elif isinstance(a, dict) and "array" in a:
                args.append(arr[a["array"]])
            else:
                args.append(a)
        out = getattr(ops, call["fn"])(*args)
        rec = call["out"]
        if rec is None:
            continue
        if "tensor" in rec:
            live[rec["tensor"]] = out
            got, want = ops.gputensor_to_numpy(out), arr[rec["value"]]
        else:
            got, want = np.asarray(out), arr[rec["array"]]
        what = f"call {i} {call['fn']}"
        assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
        assert got.dtype == want.dtype, f"{what}: dtype {got.dtype} vs {want.dtype}"
        if call["fn"] in EXACT:
            assert np.array_equal(got, want), what
        else:
            err = O.rel_frobenius(got, want)
            assert err <= 1e-5, f"{what}: rel Frobenius {err:.2e}"
