"""Seeded synthetic MoE layers in the blob format, for tests and benchmarks.

There is no checkpoint to load in this environment, so layers are generated
with the value distributions the benchmark configurations state:
  * expert codes uniform in -8..7 (stored q = code + 8, i.e. uniform bytes);
  * fp16 scales 0.01 * |N(0,1)| + 1e-3;
  * router W fp32 ~ N(0, 1/D); shared gate vector ~ N(0, 1/D);
  * optional routing skew: per-expert logit bias ln(r^-s / H) with the rank r
    of each expert drawn from a seeded permutation (so hot experts do not
    all sit at low indices).
Activations are bf16 N(0,1).

`HostLayer` holds numpy arrays (CPU); `device_layer` builds the same layout
directly in GPU memory with torch (for the full-size benchmark stacks).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

GROUP = 32

CONFIGS = {
    # name: (D, F, E, K, act, shared_f)   act 0 = GeGLU (gelu tanh), 1 = SwiGLU
    "tiny": (512, 256, 16, 4, 1, 0),
    "gemma": (2816, 704, 128, 8, 0, 0),
    "qwen": (2048, 512, 256, 8, 1, 512),
    # Gemma-like with its dense MLP branch (a shared int4 MLP of width 2112)
    "gemma_dense": (2816, 704, 128, 8, 0, 2112),
}


def blob_layout(d: int, f: int, align: int = 16):
    """Byte offsets of gate/up/down codes and scales inside one expert blob
    (MoEExpertOffsets order; bias offsets alias the scales) and the stride."""
    def up(x):
        return (x + align - 1) // align * align
    off = 0
    out = {}
    for name, rows, cols in (("gate", f, d), ("up", f, d), ("down", d, f)):
        out[name + "_w"] = off
        off = up(off + rows * cols // 2)
        out[name + "_s"] = off
        off = up(off + rows * (cols // GROUP) * 2)
    offsets = (out["gate_w"], out["gate_s"], out["gate_s"], out["up_w"], out["up_s"],
               out["up_s"], out["down_w"], out["down_s"], out["down_s"])
    return offsets, up(off)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even bf16 bits (Quantization.bf16Bits, Quantization.swift:63-69)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint32) << 16).view(np.float32)


def zipf_bias(num_experts: int, s: float, rng: np.random.Generator) -> np.ndarray:
    ranks = rng.permutation(num_experts) + 1
    h = float(np.sum(np.arange(1, num_experts + 1, dtype=np.float64) ** -s))
    return (np.log(ranks.astype(np.float64) ** -s / h)).astype(np.float32)


@dataclass
class HostLayer:
    d: int
    f: int
    num_experts: int
    top_k: int
    act: int
    experts: np.ndarray            # uint8 [E * stride]
    expert_stride: int
    offsets: tuple
    router_w: np.ndarray           # f32 [E, D]
    effective_scale: np.ndarray | None = None
    per_expert_scale: np.ndarray | None = None
    logit_bias: np.ndarray | None = None
    router_norm: bool = True
    norm_eps: float = 1e-6
    shared: np.ndarray | None = None
    shared_f: int = 0
    shared_offsets: tuple | None = None
    shared_gate: np.ndarray | None = None
    meta: dict = field(default_factory=dict)


def _fill_blob(blob: np.ndarray, offsets, d: int, f: int, rng: np.random.Generator) -> None:
    gw, gs, _, uw, us, _, dw, ds, _ = offsets
    for w_off, s_off, rows, cols in ((gw, gs, f, d), (uw, us, f, d), (dw, ds, d, f)):
        n_codes = rows * cols // 2
        blob[w_off:w_off + n_codes] = rng.integers(0, 256, n_codes, dtype=np.uint8)
        n_s = rows * (cols // GROUP)
        sc = (0.01 * np.abs(rng.standard_normal(n_s)) + 1e-3).astype(np.float16)
        blob[s_off:s_off + 2 * n_s] = sc.view(np.uint8)


def host_layer(config: str | tuple, seed: int, skew: float | None = None,
               top_k: int | None = None) -> HostLayer:
    d, f, e, k, act, shared_f = CONFIGS[config] if isinstance(config, str) else config
    if top_k is not None:
        k = top_k
    rng = np.random.default_rng(seed)
    offsets, stride = blob_layout(d, f)
    experts = np.zeros(e * stride, np.uint8)
    for i in range(e):
        _fill_blob(experts[i * stride:(i + 1) * stride], offsets, d, f, rng)
    router_w = (rng.standard_normal((e, d)) / np.sqrt(d)).astype(np.float32)
    layer = HostLayer(d=d, f=f, num_experts=e, top_k=k, act=act, experts=experts,
                      expert_stride=stride, offsets=offsets, router_w=router_w)
    if shared_f:
        so, sstride = blob_layout(d, shared_f)
        shared = np.zeros(sstride, np.uint8)
        _fill_blob(shared, so, d, shared_f, rng)
        layer.shared, layer.shared_f, layer.shared_offsets = shared, shared_f, so
        if shared_f == f:  # a shared expert is gated; a dense branch is not
            layer.shared_gate = (rng.standard_normal(d) / np.sqrt(d)).astype(np.float32)
    if skew:
        layer.logit_bias = zipf_bias(e, skew, rng)
    return layer


def host_tokens(T: int, d: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits(rng.standard_normal((T, d)).astype(np.float32))


# ---------------------------------------------------------------------------
# device-side generation (torch), same layout and distributions
# ---------------------------------------------------------------------------
def device_layer_tensors(config: str | tuple, seed: int, skew: float | None, device):
    """Returns a dict of torch tensors for one layer generated on `device`."""
    import torch

    d, f, e, k, act, shared_f = CONFIGS[config] if isinstance(config, str) else config
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    offsets, stride = blob_layout(d, f)
    experts = torch.zeros(e * stride, dtype=torch.uint8, device=device)
    ev = experts.view(e, stride)
    gw, gs, _, uw, us, _, dw, ds, _ = offsets
    for w_off, s_off, rows, cols in ((gw, gs, f, d), (uw, us, f, d), (dw, ds, d, f)):
        n_codes = rows * cols // 2
        ev[:, w_off:w_off + n_codes] = torch.randint(0, 256, (e, n_codes), generator=g,
                                                      device=device, dtype=torch.uint8)
        n_s = rows * (cols // GROUP)
        sc = (0.01 * torch.randn((e, n_s), generator=g, device=device).abs() + 1e-3).half()
        ev[:, s_off:s_off + 2 * n_s] = sc.view(torch.uint8)
    out = {
        "d": d, "f": f, "num_experts": e, "top_k": k, "act": act,
        "experts": experts, "expert_stride": stride, "offsets": offsets,
        "router_w": torch.randn((e, d), generator=g, device=device) / float(np.sqrt(d)),
    }
    if shared_f:
        so, sstride = blob_layout(d, shared_f)
        sh = torch.empty(sstride, dtype=torch.uint8, device=device)
        sgw, sgs, _, suw, sus, _, sdw, sds, _ = so
        for w_off, s_off, rows, cols in ((sgw, sgs, shared_f, d), (suw, sus, shared_f, d),
                                         (sdw, sds, d, shared_f)):
            n_codes = rows * cols // 2
            sh[w_off:w_off + n_codes] = torch.randint(0, 256, (n_codes,), generator=g,
                                                      device=device, dtype=torch.uint8)
            n_s = rows * (cols // GROUP)
            sc = (0.01 * torch.randn(n_s, generator=g, device=device).abs() + 1e-3).half()
            sh[s_off:s_off + 2 * n_s] = sc.view(torch.uint8)
        out.update(shared=sh, shared_f=shared_f, shared_offsets=so)
        if shared_f == f:  # a shared expert is gated; a dense branch is not
            out["shared_gate"] = torch.randn(d, generator=g, device=device) / float(np.sqrt(d))
    if skew:
        rng = np.random.default_rng(seed + 0x5EED)
        out["logit_bias"] = torch.from_numpy(zipf_bias(e, skew, rng)).to(device)
    return out


def to_host_layer(t: dict, experts_subset=None) -> HostLayer:
    """Copies a device layer (device_layer_tensors) back into a HostLayer."""
    layer = HostLayer(
        d=t["d"], f=t["f"], num_experts=t["num_experts"], top_k=t["top_k"], act=t["act"],
        experts=t["experts"].cpu().numpy(), expert_stride=t["expert_stride"],
        offsets=t["offsets"], router_w=t["router_w"].float().cpu().numpy())
    if "shared" in t:
        layer.shared = t["shared"].cpu().numpy()
        layer.shared_f = t["shared_f"]
        layer.shared_offsets = t["shared_offsets"]
        if t.get("shared_gate") is not None:
            layer.shared_gate = t["shared_gate"].float().cpu().numpy()
    if "logit_bias" in t:
        layer.logit_bias = t["logit_bias"].cpu().numpy()
    return layer
