"""Generates the golden fixtures in this folder from the reference itself.

Runs Tsugumi's own numpy MoE forward, ReferenceModel._moe
(Scripts/qwen35/reference_forward.py:300-334 in the reference project), on
seeded synthetic layers from tsugumi_b200.synthetic, and stores its router
choice and block output.  The reference project must be importable: its
root is read from the TSUGUMI_REFERENCE environment variable, which must be
set (there is no default).  It is only needed to regenerate the fixtures,
never at test time.

    TSUGUMI_REFERENCE=<reference checkout> python tests/golden/make_golden.py [names...]

The GeGLU fixtures run the same ``_moe`` with the module's ``silu`` replaced
by the GeGLU activation of the reference's Swift CPU reference,
``MoeRef.geluTanh`` (Sources/TsugumiValidation/Support/Reference/MoE/
Moe.swift:21-29): the numpy forward is written for Qwen (SwiGLU), and this
keeps its routing, dequantisation and combine while giving the Gemma form of
the activation.

Each fixture holds the generation parameters (config, seeds) so the tests can
rebuild the identical inputs with numpy.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tsugumi_b200.synthetic import GROUP, bf16_bits_to_f32, host_layer, host_tokens  # noqa: E402


def reference_root() -> Path:
    root = os.environ.get("TSUGUMI_REFERENCE")
    if not root:
        raise SystemExit("set TSUGUMI_REFERENCE to the reference project's root")
    path = Path(root)
    if not (path / "Scripts" / "qwen35" / "reference_forward.py").exists():
        raise SystemExit(f"{path} does not hold Scripts/qwen35/reference_forward.py")
    return path

CASES = [
    # name, (D, F, E, K, act, shared_f), layer seed, token seed, T
    ("tiny_swiglu", (512, 256, 16, 4, 1, 0), 1234, 0, 16),
    ("tiny_shared", (512, 256, 16, 4, 1, 256), 77, 0, 16),
    ("small_qwenlike", (1024, 256, 32, 8, 1, 256), 2024, 5, 24),
    # GeGLU (Gemma form): a small layer and the full Gemma-like shape
    ("small_gemmalike_geglu", (1024, 256, 32, 8, 0, 0), 31, 6, 16),
    ("gemma_geglu", (2816, 704, 128, 8, 0, 0), 4099, 9, 2),
]


def gelu_tanh(x):
    """MoeRef.geluTanh (Moe.swift:21-29), no clamp."""
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def dequant(blob: np.ndarray, w_off: int, s_off: int, rows: int, cols: int) -> np.ndarray:
    codes = blob[w_off:w_off + rows * cols // 2].reshape(rows, cols // 2)
    q = np.empty((rows, cols), np.float32)
    q[:, 0::2] = (codes & 0x0F).astype(np.float32)
    q[:, 1::2] = (codes >> 4).astype(np.float32)
    s = blob[s_off:s_off + rows * (cols // GROUP) * 2].view(np.float16).astype(np.float32)
    s = s.reshape(rows, cols // GROUP)
    return ((q.reshape(rows, cols // GROUP, GROUP) - 8.0) * s[:, :, None]).reshape(rows, cols)


def reference_moe(layer, xn: np.ndarray):
    sys.path.insert(0, str(reference_root() / "Scripts" / "qwen35"))
    import reference_forward as rf  # the reference's own module

    rf_silu = rf.silu
    if layer.act == 0:
        rf.silu = gelu_tanh
    try:
        return _run_reference_moe(rf, layer, xn)
    finally:
        rf.silu = rf_silu


def _run_reference_moe(rf, layer, xn: np.ndarray):
    d, f = layer.d, layer.f
    gw, gs, _, uw, us, _, dw, ds, _ = layer.offsets
    stride = layer.expert_stride

    def expert_w(e, which):
        blob = layer.experts[e * stride:(e + 1) * stride]
        if which == "gate":
            return dequant(blob, gw, gs, f, d)
        if which == "up":
            return dequant(blob, uw, us, f, d)
        return dequant(blob, dw, ds, d, f)

    p = "L"
    mats = {f"{p}.gate": layer.router_w.astype(np.float32)}
    if layer.shared is not None:
        so = layer.shared_offsets
        sf = layer.shared_f
        mats[f"{p}.shared_expert.gate_proj"] = dequant(layer.shared, so[0], so[1], sf, d)
        mats[f"{p}.shared_expert.up_proj"] = dequant(layer.shared, so[3], so[4], sf, d)
        mats[f"{p}.shared_expert.down_proj"] = dequant(layer.shared, so[6], so[7], d, sf)
        mats[f"{p}.shared_expert_gate"] = layer.shared_gate.reshape(1, d)
    else:  # the reference always adds the shared branch: give it zero weights
        mats[f"{p}.shared_expert.gate_proj"] = np.zeros((f, d), np.float32)
        mats[f"{p}.shared_expert.up_proj"] = np.zeros((f, d), np.float32)
        mats[f"{p}.shared_expert.down_proj"] = np.zeros((d, f), np.float32)
        mats[f"{p}.shared_expert_gate"] = np.zeros((1, d), np.float32)

    stub = types.SimpleNamespace()
    stub.cfg = types.SimpleNamespace(top_k=layer.top_k)
    stub.bytes_dequantized = 0
    stub._dense = lambda x, name: x @ mats[name].T
    names = {"gate_proj": "gate", "up_proj": "up", "down_proj": "down"}
    stub.deq = types.SimpleNamespace(
        slice3=lambda name, e: expert_w(e, names[name.rsplit(".", 1)[1]]))
    dump: dict = {}
    y = rf.ReferenceModel._moe(stub, xn.astype(np.float32), 0, dump, prefix=p)
    return y.astype(np.float32), dump["layer0.router_idx"], dump["layer0.router_w"]


def main(only: list[str]) -> None:
    for name, cfg, lseed, tseed, T in CASES:
        if only and name not in only:
            continue
        layer = host_layer(cfg, lseed)
        x = host_tokens(T, cfg[0], tseed)
        xf = bf16_bits_to_f32(x).astype(np.float64)
        inv = 1.0 / np.sqrt(np.mean(xf * xf, axis=1, keepdims=True) + 1e-6)
        xn = (xf * inv).astype(np.float32)  # the block input after the no-scale RMSNorm
        y, idx, w = reference_moe(layer, xn)
        np.savez_compressed(HERE / f"{name}.npz", config=np.array(cfg), layer_seed=lseed,
                            token_seed=tseed, T=T, y=y, router_idx=idx.astype(np.int32),
                            router_w=w.astype(np.float32))
        print(name, y.shape, float(np.abs(y).max()))


if __name__ == "__main__":
    main(sys.argv[1:])  # optional fixture names: regenerate only those
