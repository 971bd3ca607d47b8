"""A numpy restatement of the reference's MoE block (second CPU reference).

TEST INFRASTRUCTURE ONLY, like the rest of oracle/: used by tests/ (as a
second, independent restatement checked against the C oracle and the golden
fixtures) and by bench.py's CPU-baseline leg (timed on the Qwen-like
config).  The product path never imports it.

It follows two reference sources:

* the reference's numpy forward, ``ReferenceModel._moe``
  (Scripts/qwen35/reference_forward.py:300-334): fp32 router logits, softmax
  over all experts, top-K, renormalised weights; for each distinct expert the
  int4 matrices are dequantised for the call (``deq.slice3``) and applied as
  ``act(x Wg^T) * (x Wu^T)`` then ``Wd``; the shared expert is gated by
  ``sigmoid(x . w_s)``;
* the Swift CPU reference ``MoeRef`` (Sources/TsugumiValidation/Support/
  Reference/MoE/Moe.swift:16-56) for the GeGLU form of the activation,
  ``0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))`` with no clamp.

Dequantisation is ``Quantization.dequantizeInt4Affine`` for the symmetric
scheme (Quantization.swift:210-227): ``q * s + b`` with ``b = -8 s``, i.e.
``s (q - 8)``.  Top-K ties go to the lower expert index, as in
RouterTopKTests.swift:270-295 (the numpy forward's ``argpartition`` leaves
ties unordered, so tests exclude near-ties).

The block input is the no-scale RMSNorm of the bf16 hidden rows when the
layer asks for it (rmsnorm.metal:154-175), computed in fp64 and rounded to
fp32, as tests/golden/make_golden.py does for the reference's own ``_moe``.

``gemma_ffn`` restates Gemma's layer FFN with the norms and residuals the
reference fuses around the block (fused.metal:190-374).
"""

from __future__ import annotations

import numpy as np

GROUP = 32
GELU_C = 0.7978845608028654
GELU_K = 0.044715


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """MoeRef.geluTanh (Moe.swift:21-29)."""
    return 0.5 * x * (1.0 + np.tanh(GELU_C * (x + GELU_K * x * x * x)))


def silu(x: np.ndarray) -> np.ndarray:
    """reference_forward.silu: x / (1 + e^-x)."""
    return x / (1.0 + np.exp(-x))


def sigmoid(x: np.ndarray) -> np.ndarray:
    return 1.0 / (1.0 + np.exp(-x))


def dequant(blob: np.ndarray, w_off: int, s_off: int, rows: int, cols: int) -> np.ndarray:
    """One int4 symmetric group-32 matrix of a blob as fp32 [rows, cols]:
    low nibble = even element, fp16 scale per 32 columns, w = s (q - 8)."""
    codes = blob[w_off:w_off + rows * cols // 2].reshape(rows, cols // 2)
    q = np.empty((rows, cols), np.float32)
    q[:, 0::2] = codes & 0x0F
    q[:, 1::2] = codes >> 4
    s = blob[s_off:s_off + rows * (cols // GROUP) * 2].view(np.float16).astype(np.float32)
    s = s.reshape(rows, cols // GROUP, 1)
    return ((q.reshape(rows, cols // GROUP, GROUP) - 8.0) * s).reshape(rows, cols)


def normalise(layer, x_bf16: np.ndarray) -> np.ndarray:
    """The block input: bf16 rows, no-scale RMSNorm'd when router_norm."""
    xf = (np.asarray(x_bf16, np.uint32) << 16).view(np.float32).astype(np.float64)
    if not layer.router_norm:
        return xf.astype(np.float32)
    inv = 1.0 / np.sqrt(np.mean(xf * xf, axis=1, keepdims=True) + layer.norm_eps)
    return (xf * inv).astype(np.float32)


def route(layer, xn: np.ndarray):
    """fp32 logits, softmax over all experts, top-K (larger first, ties to
    the lower index), renormalised: reference_forward.py:306-313."""
    w = layer.router_w.astype(np.float32)
    if layer.effective_scale is not None:
        w = w * layer.effective_scale[None, :].astype(np.float32)
    logits = xn @ w.T
    if layer.logit_bias is not None:
        logits = logits + layer.logit_bias[None, :]
    z = logits - logits.max(axis=1, keepdims=True)
    probs = np.exp(z)
    probs /= probs.sum(axis=1, keepdims=True)
    k = layer.top_k
    e = probs.shape[1]
    # lexsort: last key is primary -> (-prob, index)
    order = np.lexsort((np.broadcast_to(np.arange(e), probs.shape), -probs), axis=1)[:, :k]
    vals = np.take_along_axis(probs, order, axis=1)
    weights = vals / vals.sum(axis=1, keepdims=True)
    if layer.per_expert_scale is not None:
        weights = weights * layer.per_expert_scale[order]
    return order.astype(np.uint32), weights.astype(np.float32), logits


def ffn(blob: np.ndarray, offsets, d: int, f: int, x: np.ndarray, act: int) -> np.ndarray:
    """down(act(gate x) * up x) for the rows x [n, d] (Moe.swift:33-56,
    reference_forward.py:324-326)."""
    gw, gs, _, uw, us, _, dw, ds, _ = offsets
    wg = dequant(blob, gw, gs, f, d)
    wu = dequant(blob, uw, us, f, d)
    wd = dequant(blob, dw, ds, d, f)
    g = x @ wg.T
    h = (gelu_tanh(g) if act == 0 else silu(g)) * (x @ wu.T)
    return h @ wd.T


def moe_block(layer, x_bf16: np.ndarray, ids: np.ndarray | None = None,
              weights: np.ndarray | None = None) -> np.ndarray:
    """y = sum_k w_k expert_k(x) (+ sigmoid(x . w_s) shared(x)), fp32, for
    a synthetic.HostLayer; routing from the router unless given."""
    xn = normalise(layer, x_bf16)
    if ids is None:
        ids, weights, _ = route(layer, xn)
    stride = layer.expert_stride
    y = np.zeros_like(xn)
    for expert in np.unique(ids):
        rows, slots = np.nonzero(ids == expert)
        blob = layer.experts[int(expert) * stride:(int(expert) + 1) * stride]
        out = ffn(blob, layer.offsets, layer.d, layer.f, xn[rows], layer.act)
        y[rows] += weights[rows, slots][:, None] * out
    if layer.shared is not None:
        sh = ffn(layer.shared, layer.shared_offsets, layer.d, layer.shared_f, xn, layer.act)
        if layer.shared_gate is not None:
            sh = sigmoid(xn @ layer.shared_gate.astype(np.float32))[:, None] * sh
        y = y + sh
    return y.astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 -> fp32, round to nearest even."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint32) << 16).view(np.float32)


def _inv_rms(x: np.ndarray, eps: float) -> np.ndarray:
    x64 = x.astype(np.float64)
    return (1.0 / np.sqrt(np.mean(x64 * x64, axis=1, keepdims=True) + eps)).astype(np.float32)


def gemma_ffn(layer, norms: dict, hidden_bf16: np.ndarray, attn_bf16: np.ndarray,
              eps: float, layer_scalar: float) -> np.ndarray:
    """Gemma's layer FFN with the adjacent norms: fused_post_attn_setup and
    fused_layer_tail (Sources/Tsugumi/Metal/Fusions/fused.metal:190-267,
    :269-374) around the dense branch (SharedExpertInt4.swift:30-94, then
    its post-norm, RealForwardRunner.swift:3236-3242) and the routed block
    (routed on the normalised row, experts on it times pre_ffn2).  RMSNorm is
    x * rsqrt(mean(x^2) + eps) * w; every stored intermediate is rounded to
    bf16 where the reference rounds to fp16.  `norms` holds bf16 bit arrays
    [D]; `layer` is a HostLayer whose shared blob is the dense branch.
    Returns the new hidden rows (fp32 values, bf16-representable)."""
    import copy

    w = {k: bf16_bits_to_f32(v)[None, :] for k, v in norms.items()}
    h0 = bf16_bits_to_f32(hidden_bf16)
    a = bf16_bits_to_f32(attn_bf16)
    a_n = bf16_round(a * _inv_rms(a, eps) * w["post_attn"])
    h = bf16_round(h0 + a_n)
    xh = h * _inv_rms(h, eps)
    router_x = bf16_round(xh)
    routed_x = bf16_round(xh * w["pre_ffn2"])
    dense_x = bf16_round(xh * w["pre_ffn"])
    routed = copy.copy(layer)
    routed.router_norm = False
    routed.shared = None
    to_bits = lambda v: (v.view(np.uint32) >> 16).astype(np.uint16)  # noqa: E731
    ids, weights, _ = route(routed, router_x)
    h2 = moe_block(routed, to_bits(routed_x), ids, weights)
    r = bf16_round(h2 * _inv_rms(h2, eps) * w["post_routed"])
    if layer.shared is not None:
        h1 = ffn(layer.shared, layer.shared_offsets, layer.d, layer.shared_f, dense_x, layer.act)
        d1 = bf16_round(h1.astype(np.float32) * _inv_rms(h1, eps) * w["post_dense"])
    else:
        d1 = np.zeros_like(r)
    h12 = bf16_round(d1 + r)
    f = bf16_round(h12 * _inv_rms(h12, eps) * w["post_ffn"])
    scale = bf16_round(np.array([layer_scalar], np.float32))[0]
    return bf16_round(bf16_round(h + f) * scale), h
