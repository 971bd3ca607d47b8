"""The .moepack reader: layout validation (CPU) and the exact device import
of expert blobs with BF16 scales (GPU).

The validation cases follow MoEPackV1StructuralValidator.validate
(MoEPackPackedExpertsLayoutV1.swift:88-172); the import is checked bit for
bit against the blob it was written from, and through a block forward
against the oracle."""

from __future__ import annotations

import copy
import json
from pathlib import Path

import numpy as np
import pytest

from tsugumi_b200 import moepack as mp
from tsugumi_b200.synthetic import blob_layout, host_layer, host_tokens

STRIDE = mp.ALIGNMENT


def _layout_dict(num_layers=2, experts=4, stride=STRIDE):
    def expert(pos):
        return {"offset": pos * stride, "size": stride, "tensors": {
            "gate": {"offset": 0, "size": 4096, "dtype": "U32", "shape": [64, 16], "bits": 4},
            "gate_scales": {"offset": 4096, "size": 256, "dtype": "BF16", "shape": [64, 2]}}}
    return {"expertStride": stride, "numLayers": num_layers, "expertsPerLayer": experts,
            "layers": [{"layer": i, "file": f"layer_{i:03d}.bin",
                        "experts": [expert(p) for p in range(experts)]}
                       for i in range(num_layers)]}


def test_valid_layout_round_trips():
    lay = mp.decode_layout(json.dumps(_layout_dict()))
    assert lay.num_layers == 2 and lay.experts_per_layer == 4
    again = mp.decode_layout(mp.encode_layout(lay))
    assert again == lay
    assert lay.expert(1, 3).offset == 3 * STRIDE


def _mutations():
    def m(fn):
        d = _layout_dict()
        fn(d)
        return d
    return [
        ("layout", m(lambda d: d.update(expertStride=STRIDE + 16))),
        ("layout", m(lambda d: d.update(numLayers=3))),
        ("layout.layers", m(lambda d: d["layers"][1].update(layer=0))),
        ("layout.layers[1].file", m(lambda d: d["layers"][1].update(file="LAYER_000.bin"))),
        ("layout.layers[0].file", m(lambda d: d["layers"][0].update(file="layout.json"))),
        ("layout.layers[0].file", m(lambda d: d["layers"][0].update(file="a/b.bin"))),
        ("layout.layers[0].experts", m(lambda d: d["layers"][0]["experts"].pop())),
        ("layout.layers[0].experts", m(lambda d: d["layers"][0]["experts"][0].update(expert=0))),
        ("expert[1]", m(lambda d: d["layers"][0]["experts"][1].update(offset=5 * STRIDE))),
        ("layout.layers[0].experts",
         m(lambda d: d["layers"][0]["experts"][1].update(offset=0))),
        ("expert[0].tensors.gate",
         m(lambda d: d["layers"][0]["experts"][0]["tensors"]["gate"].update(dtype="F16"))),
        ("expert[0].tensors.gate",
         m(lambda d: d["layers"][0]["experts"][0]["tensors"]["gate"].update(bits=33))),
        ("expert[0].tensors.gate_scales",
         m(lambda d: d["layers"][0]["experts"][0]["tensors"]["gate_scales"].update(
             offset=STRIDE - 100))),
        ("expert[0].tensors",
         m(lambda d: d["layers"][0]["experts"][0]["tensors"]["gate_scales"].update(offset=4000))),
    ]


@pytest.mark.parametrize("field,data", _mutations())
def test_invalid_layouts_are_rejected(field, data):
    with pytest.raises(mp.MoEPackFormatError) as exc:
        mp.decode_layout(json.dumps(data))
    assert exc.value.field == field


def test_malformed_json_is_a_format_error():
    with pytest.raises(mp.MoEPackFormatError):
        mp.decode_layout(b'{"expertStride": 16384')


# ---------------------------------------------------------------------------
# writing a .moepack from a synthetic layer (test fixture)

def _bf16_representable_scales(host, groups64=()):
    """Rounds every fp16 scale of the layer's blobs to a value with at most 8
    significant bits (a BF16 value, still exact in fp16); for the roles in
    groups64 each pair of 32-groups gets one scale (a 64-group)."""
    offs = host.offsets
    names = ("gate", "up", "down")
    for e in range(host.num_experts):
        blob = host.experts[e * host.expert_stride:(e + 1) * host.expert_stride]
        for i, role in enumerate(names):
            rows, cols = (host.f, host.d) if role != "down" else (host.d, host.f)
            s_off = offs[3 * i + 1]
            n = rows * cols // 32
            sc = blob[s_off:s_off + 2 * n].view(np.float16).astype(np.float32)
            bits = sc.view(np.uint32)
            bits = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
            sc = bits.view(np.float32).reshape(rows, cols // 32)
            if role in groups64:
                sc[:, 1::2] = sc[:, 0::2]
            blob[s_off:s_off + 2 * n] = sc.astype(np.float16).reshape(-1).view(np.uint8)


def write_moepack(root: Path, host, groups64=(), biases=()):
    """One layer of `host` as a .moepack: U32 codes (the same bytes), BF16
    scales per 32- or 64-group, BF16 biases -8 x scale for the roles in
    `biases`, tensors 256-byte aligned in 16 KiB-aligned expert blobs."""
    offs = host.offsets
    tensors, cur = [], 0
    for i, role in enumerate(("gate", "up", "down")):
        rows, cols = (host.f, host.d) if role != "down" else (host.d, host.f)
        g = 64 if role in groups64 else 32
        parts = [(role, rows * cols // 2, "U32", [rows, cols // 8], 4),
                 (f"{role}_scales", rows * (cols // g) * 2, "BF16", [rows, cols // g], None)]
        if role in biases:
            parts.append((f"{role}_biases", rows * (cols // g) * 2, "BF16", [rows, cols // g], None))
        for name, size, dt, shape, bits in parts:
            cur = (cur + 255) // 256 * 256
            tensors.append((name, cur, size, dt, shape, bits, role, i, g))
            cur += size
    stride = (cur + STRIDE - 1) // STRIDE * STRIDE
    E = host.num_experts
    data = np.zeros(E * stride, np.uint8)
    experts = []
    for e in range(E):
        phys = (e * 5 + 3) % E if E % 5 else e  # physical ranks permuted
        blob = host.experts[e * host.expert_stride:(e + 1) * host.expert_stride]
        dst = data[phys * stride:(phys + 1) * stride]
        tj = {}
        for name, off, size, dt, shape, bits, role, i, g in tensors:
            rows, cols = shape[0], (shape[1] * 8 if dt == "U32" else shape[1] * g)
            if dt == "U32":
                dst[off:off + size] = blob[offs[3 * i]:offs[3 * i] + size]
            else:
                s16 = blob[offs[3 * i + 1]:offs[3 * i + 1] + rows * cols // 16].view(np.float16)
                s = s16.astype(np.float32).reshape(rows, cols // 32)[:, ::g // 32]
                sb = (s.view(np.uint32) >> 16).astype(np.uint16)
                if name.endswith("_biases"):
                    v = (sb.astype(np.uint32) << 16).view(np.float32) * np.float32(-8)
                    b = v.view(np.uint32)
                    sb = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
                dst[off:off + size] = sb.reshape(-1).view(np.uint8)
            tj[name] = {"offset": off, "size": size, "dtype": dt, "shape": shape}
            if bits:
                tj[name]["bits"] = bits
        experts.append({"expert": e, "physicalRank": phys, "offset": phys * stride,
                        "size": stride, "tensors": tj})
    lay = {"expertStride": stride, "numLayers": 1, "expertsPerLayer": E,
           "layers": [{"layer": 0, "file": "layer_000.bin", "experts": experts}]}
    pe = root / "packed_experts"
    pe.mkdir(parents=True, exist_ok=True)
    (pe / "layout.json").write_text(json.dumps(lay))
    data.tofile(pe / "layer_000.bin")
    return stride


@pytest.mark.gpu
@pytest.mark.parametrize("groups64,biases", [((), ()), (("down",), ("gate",)),
                                            (("gate", "up", "down"), ("gate", "up", "down"))])
def test_import_is_exact_and_runs(tmp_path, groups64, biases):
    torch = pytest.importorskip("torch")
    import tsugumi_b200 as tb
    from oracle import oracle as O

    host = host_layer("tiny", 31)
    _bf16_representable_scales(host, groups64)
    write_moepack(tmp_path, host, groups64, biases)
    ctx = tb.Context(0)
    layout = mp.read_layout(tmp_path)
    t = mp.import_layer(ctx, tmp_path, layout, 0, host.d, host.f)
    assert t["expert_stride"] == host.expert_stride and tuple(t["offsets"]) == tuple(host.offsets)
    assert np.array_equal(t["experts"].cpu().numpy(), host.experts)  # bit for bit
    tensors = tb.upload_host_layer(host)
    tensors.update(t)
    layer = tb.MoELayer(ctx, tensors)
    x = host_tokens(16, host.d, 3)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
    y = layer.forward(xd, out_dtype=torch.float32)
    ctx.sync()
    ids = torch.empty((16, host.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((16, host.top_k), dtype=torch.float32, device="cuda")
    tb.MoE(ctx, layer).encode_router_gemma4_bf16(xd, ids, w)
    ctx.sync()
    y_ref, _, _ = O.OracleLayer(host).block(x, ids.cpu().numpy().astype(np.uint32), w.cpu().numpy())
    err = np.linalg.norm(y.cpu().numpy() - y_ref) / np.linalg.norm(y_ref)
    assert err <= 2e-3


@pytest.mark.gpu
def test_import_rejects_inexact_scale_and_asymmetric_bias(tmp_path):
    pytest.importorskip("torch")
    import tsugumi_b200 as tb

    host = host_layer("tiny", 32)
    _bf16_representable_scales(host)
    write_moepack(tmp_path / "a", host, (), ("gate",))
    layout = mp.read_layout(tmp_path / "a")
    ctx = tb.Context(0)
    f = tmp_path / "a" / "packed_experts" / "layer_000.bin"
    raw = np.fromfile(f, np.uint8)
    e0 = layout.expert(0, 0)
    good = raw.copy()
    # a BF16 scale below fp16's range (2^-30): representable in BF16, not fp16
    so = e0.offset + e0.tensors["up_scales"].offset
    raw[so:so + 2] = np.array([0x3080], np.uint16).view(np.uint8)
    raw.tofile(f)
    with pytest.raises(mp.MoEPackFormatError) as exc:
        mp.import_layer(ctx, tmp_path / "a", layout, 0, host.d, host.f)
    assert "not an fp16 value" in str(exc.value)
    # a bias that is not -8 x scale (an affine, not symmetric, blob)
    raw = good.copy()
    bo = e0.offset + e0.tensors["gate_biases"].offset
    raw[bo:bo + 2] ^= np.array([1, 0], np.uint8)
    raw.tofile(f)
    with pytest.raises(mp.MoEPackFormatError) as exc:
        mp.import_layer(ctx, tmp_path / "a", layout, 0, host.d, host.f)
    assert "not -8 x scale" in str(exc.value)
