"""Generate golden vectors by running the REFERENCE's own CPU code.

Usage (in a container that has the reference tree; not needed at test time)::

    python tests/golden/make_golden.py /path/to/reference

The reference package is copied to a temporary directory and imported as
``scaffolding``.  With no compiled extensions present its CPU path is
NumPy/OpenBLAS (``tensor.py:20-41``), i.e. exactly the code the oracle
restates.  Each case below calls the reference's public API
(``nn.Linear``, ``F.silu``, ``F.gelu``, ``F.linear``, ``F.softmax``,
``sf.matmul``, ``sf.matmul_nt``, ``F.scaled_dot_product_attention``,
``nn.LayerNorm`` / ``diffusion.models.AdaLayerNorm`` and
``CrossAttentionBlock._attn``) on seeded
inputs and stores inputs + outputs in ``golden.npz`` next to this script.
Config 1 (512x1024 -> 4096, SiLU) is too large to store whole: its inputs are
regenerated from the seed and a row subsample plus full-array checksums of
the output are stored.
"""
from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

CONFIG1_ROW_STRIDE = 8


def _import_reference(ref_root: str):
    tmp = tempfile.mkdtemp(prefix="sf_ref_")
    shutil.copytree(ref_root, os.path.join(tmp, "scaffolding"),
                    ignore=shutil.ignore_patterns("*.so", "build", "*.egg-info"))
    sys.path.insert(0, tmp)
    import importlib
    sf = importlib.import_module("scaffolding")
    T = importlib.import_module("scaffolding.tensor")
    assert not T._USE_CUDA and not T._USE_CYTHON and not T._USE_MPS, \
        "reference must run on its NumPy path"
    nn = importlib.import_module("scaffolding.nn")
    F = importlib.import_module("scaffolding.nn.functional")
    return sf, nn, F


def main(ref_root: str) -> None:
    sf, nn, F = _import_reference(ref_root)
    Tensor = sf.Tensor
    out: dict[str, np.ndarray] = {}
    meta: dict = {"numpy": np.__version__}
    try:
        cfg = np.show_config(mode="dicts")
        meta["blas"] = cfg["Build Dependencies"]["blas"]
    except Exception:  # pragma: no cover
        meta["blas"] = None
    meta["OPENBLAS_NUM_THREADS"] = os.environ.get("OPENBLAS_NUM_THREADS")

    def lin_ref(x, W, b, act):
        lin = nn.Linear(W.shape[1], W.shape[0], bias=b is not None)
        lin.weight._data = np.ascontiguousarray(W, dtype=np.float32)
        if b is not None:
            lin.bias._data = np.ascontiguousarray(b, dtype=np.float32)
        y = lin(Tensor(np.ascontiguousarray(x, dtype=np.float32)))
        if act == "silu":
            y = F.silu(y)
        elif act == "gelu_tanh":
            y = F.gelu(y)
        return np.asarray(y._data)

    # ── config 1: nn.Linear fp32 + SiLU, seed 0 (inputs regenerated from seed)
    x, W, b = O.config1_inputs(seed=0)
    y = lin_ref(x, W, b, "silu")
    out["cfg1_y_rows"] = y[::CONFIG1_ROW_STRIDE].copy()
    out["cfg1_y_sum"] = np.array(y.astype(np.float64).sum())
    out["cfg1_y_sumsq"] = np.array((y.astype(np.float64) ** 2).sum())
    out["cfg1_y_shape"] = np.array(y.shape)
    meta["cfg1_row_stride"] = CONFIG1_ROW_STRIDE

    rng = np.random.default_rng(12345)

    def rn(*shape):
        return rng.standard_normal(shape, dtype=np.float32)

    # ── small 2-D / batched matmuls (ragged shapes)
    for tag, (m, k, n) in {"mm_a": (37, 53, 29), "mm_b": (1, 8, 5),
                           "mm_c": (130, 72, 260)}.items():
        a, bb, bt = rn(m, k), rn(k, n), rn(n, k)
        out[f"{tag}_a"], out[f"{tag}_b"], out[f"{tag}_bt"] = a, bb, bt
        out[f"{tag}_nn"] = sf.matmul(Tensor(a), Tensor(bb))._data
        out[f"{tag}_nt"] = sf.matmul_nt(Tensor(a), Tensor(bt))._data

    a, bb, bt = rn(2, 3, 17, 24), rn(2, 3, 24, 19), rn(2, 3, 19, 24)
    out["bmm_a"], out["bmm_b"], out["bmm_bt"] = a, bb, bt
    out["bmm_nn"] = sf.matmul(Tensor(a), Tensor(bb))._data
    out["bmm_nt"] = sf.matmul_nt(Tensor(a), Tensor(bt))._data

    # ── linear + activations, fp32 and on bf16-rounded inputs
    for tag, (m, k, n, act, dt) in {
            "lin_silu_f32": (33, 64, 48, "silu", "f32"),
            "lin_gelu_f32": (9, 96, 80, "gelu_tanh", "f32"),
            "lin_none_f32": (5, 40, 24, "none", "f32"),
            "lin_gelu_bf16": (20, 128, 96, "gelu_tanh", "bf16"),
            "lin_silu_f16": (17, 64, 112, "silu", "f16")}.items():
        xx = O.round_to(rn(m, k), dt)
        ww = O.round_to(rn(n, k) * np.float32(0.05), dt)
        bbias = O.round_to(rn(n) * np.float32(0.05), dt)
        out[f"{tag}_x"], out[f"{tag}_w"], out[f"{tag}_b"] = xx, ww, bbias
        out[f"{tag}_y"] = lin_ref(xx, ww, bbias, act)
        # the functional form must agree with the module form
        yf = F.linear(Tensor(xx), Tensor(ww), Tensor(bbias))._data
        if act == "silu":
            yf = F.silu(Tensor(yf))._data
        elif act == "gelu_tanh":
            yf = F.gelu(Tensor(yf))._data
        out[f"{tag}_yf"] = yf

    # ── elementwise activations over a wide range
    z = np.linspace(-12, 12, 4801, dtype=np.float32)
    out["act_z"] = z
    out["act_silu"] = F.silu(Tensor(z))._data
    out["act_gelu"] = F.gelu(Tensor(z))._data

    # ── row softmax
    s1, s2 = rn(7, 300) * 4, rn(3, 1500) * 8
    out["sm1_x"], out["sm2_x"] = s1, s2
    out["sm1_y"] = F.softmax(Tensor(s1), -1)._data
    out["sm2_y"] = F.softmax(Tensor(s2), -1)._data

    # ── scaled-dot-product attention (no mask), fp32 and scale=1/8
    q, k, v = rn(2, 3, 40, 16), rn(2, 3, 56, 16), rn(2, 3, 56, 16)
    out["sdpa_q"], out["sdpa_k"], out["sdpa_v"] = q, k, v
    out["sdpa_o"] = F.scaled_dot_product_attention(Tensor(q), Tensor(k), Tensor(v))._data
    q2, k2, v2 = [O.round_bf16(rn(1, 2, 70, 64)) for _ in range(3)]
    out["sdpa8_q"], out["sdpa8_k"], out["sdpa8_v"] = q2, k2, v2
    out["sdpa8_o"] = F.scaled_dot_product_attention(
        Tensor(q2), Tensor(k2), Tensor(v2), scale=0.125)._data

    # ── LayerNorm and AdaLayerNorm (nn/layers.py:443-521, diffusion/models.py:470-487)
    import importlib
    M = importlib.import_module("scaffolding.diffusion.models")
    C, cond_dim, N = 64, 32, 24
    xa = rn(1, N, C) * np.float32(2) + np.float32(0.5)
    cond = rn(1, cond_dim)
    ada = M.AdaLayerNorm(C, cond_dim)
    ada.norm.weight._data = (1 + 0.1 * rn(C)).astype(np.float32)
    ada.norm.bias._data = (0.1 * rn(C)).astype(np.float32)
    ada.linear.weight._data = (0.05 * rn(2 * C, cond_dim)).astype(np.float32)
    ada.linear.bias._data = (0.05 * rn(2 * C)).astype(np.float32)
    out["adaln_x"], out["adaln_cond"] = xa, cond
    out["adaln_gamma"], out["adaln_beta"] = ada.norm.weight._data, ada.norm.bias._data
    out["adaln_w"], out["adaln_b"] = ada.linear.weight._data, ada.linear.bias._data
    out["adaln_params"] = ada.linear(Tensor(cond))._data
    out["adaln_ln"] = ada.norm(Tensor(xa))._data
    out["adaln_y"] = ada(Tensor(xa), Tensor(cond))._data

    # ── the DiT-family host attention CrossAttentionBlock._attn (diffusion/models.py:123-133)
    bq, bk, bv = rn(2, 3, 20, 16), rn(2, 3, 9, 16), rn(2, 3, 9, 16)
    out["battn_q"], out["battn_k"], out["battn_v"] = bq, bk, bv
    out["battn_o"] = M.CrossAttentionBlock._attn(None, bq, bk, bv)

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, default=str)
    print(f"wrote {path} ({os.path.getsize(path) / 1e6:.2f} MB, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference project root>")
    main(sys.argv[1])
