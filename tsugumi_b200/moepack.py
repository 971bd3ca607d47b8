"""The .moepack packed-experts reader.

Restates the reference's format (Sources/MoEPackFormat/
MoEPackPackedExpertsLayoutV1.swift:3-212): ``packed_experts/layout.json``
describes, per layer, a file of ``expertsPerLayer`` expert blobs of
``expertStride`` bytes each (physical rank r at offset r * stride), and per
expert its sub-tensors by name -- ``gate``, ``up``, ``down`` (U32 packed int4
codes, MLX affine layout), ``<role>_scales`` (BF16) and, unless the blob is
``sym``, ``<role>_biases`` (BF16) -- as ``ModelExpertIO.routedExpertOffsets``
(ModelExpertIO.swift:55-84) reads them.

``decode_layout`` parses and validates a layout the way
``MoEPackV1StructuralValidator.validate`` (MoEPackPackedExpertsLayoutV1.swift:
88-172) does, raising ``MoEPackFormatError`` with the same field names.
``import_layer`` reads one layer file, copies it to the device and converts
every expert's three projections into this library's blob layout there
(``tsg_import_int4_affine``: codes as bytes, fp16 scales per 32-group; exact
or an error at ``Context.sync``), giving the tensors ``MoELayer`` takes.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from ._abi import check
from .moe import PrefillMoEGroupingError

ALIGNMENT = 16384  # MoEPackFormatV1.alignmentBytes (MoEPackFormatV1.swift:24)
ROLES = ("gate", "up", "down")


class MoEPackFormatError(ValueError):
    """MoEPackFormatError.invalid(field:reason:)."""

    def __init__(self, field_name: str, reason: str):
        super().__init__(f"invalid {field_name}: {reason}")
        self.field, self.reason = field_name, reason


@dataclass
class SubTensor:
    offset: int
    size: int
    dtype: str
    shape: list
    bits: int | None = None


@dataclass
class Expert:
    offset: int
    size: int
    tensors: dict
    expert: int | None = None
    physical_rank: int | None = None


@dataclass
class Layer:
    layer: int
    file: str
    experts: list = field(default_factory=list)


@dataclass
class Layout:
    expert_stride: int
    num_layers: int
    experts_per_layer: int
    layers: list

    def expert(self, layer: int, logical: int) -> Expert:
        """The expert with logical id ``logical`` of layer ``layer``."""
        lay = next(x for x in self.layers if x.layer == layer)
        for pos, e in enumerate(lay.experts):
            if (e.expert if e.expert is not None else pos) == logical:
                return e
        raise KeyError(logical)


def _validate_basename(name: str, field_name: str) -> None:
    # MoEPackPathValidator.validateBasename: a plain file name
    if (not name or name in (".", "..") or "/" in name or "\\" in name or "\x00" in name):
        raise MoEPackFormatError(field_name, "not a plain file name")


def validate(layout: Layout) -> None:
    """MoEPackV1StructuralValidator.validate (MoEPackPackedExpertsLayoutV1.swift:88-172)."""
    if not (layout.num_layers > 0 and layout.experts_per_layer > 0 and layout.expert_stride > 0
            and layout.expert_stride % ALIGNMENT == 0
            and len(layout.layers) == layout.num_layers):
        raise MoEPackFormatError("layout", "invalid dimensions or stride")
    layer_ids, files = set(), set()
    for lay in layout.layers:
        if not (0 <= lay.layer < layout.num_layers) or lay.layer in layer_ids:
            raise MoEPackFormatError("layout.layers", "duplicate or invalid layer")
        layer_ids.add(lay.layer)
        _validate_basename(lay.file, f"layout.layers[{lay.layer}].file")
        key = lay.file.lower()  # the Apple file system compares names without case
        if key == "layout.json":
            raise MoEPackFormatError(f"layout.layers[{lay.layer}].file",
                                     "reserved packed-expert filename")
        if key in files:
            raise MoEPackFormatError(f"layout.layers[{lay.layer}].file", "duplicate layer filename")
        files.add(key)
        if len(lay.experts) != layout.experts_per_layer:
            raise MoEPackFormatError(f"layout.layers[{lay.layer}].experts", "wrong expert count")
        explicit = [e.expert is not None for e in lay.experts]
        if any(explicit) and not all(explicit):
            raise MoEPackFormatError(f"layout.layers[{lay.layer}].experts",
                                     "expert ids must be either all explicit or all positional")
        logical_ids, physical_ranks, offsets = set(), set(), set()
        for pos, e in enumerate(lay.experts):
            logical = e.expert if e.expert is not None else pos
            physical = e.physical_rank if e.physical_rank is not None else logical
            if not (0 <= logical < layout.experts_per_layer
                    and 0 <= physical < layout.experts_per_layer
                    and logical not in logical_ids and physical not in physical_ranks
                    and e.offset not in offsets):
                raise MoEPackFormatError(f"layout.layers[{lay.layer}].experts",
                                         "duplicate or invalid expert mapping")
            logical_ids.add(logical)
            physical_ranks.add(physical)
            offsets.add(e.offset)
            if e.offset != physical * layout.expert_stride or e.size != layout.expert_stride:
                raise MoEPackFormatError(f"expert[{logical}]",
                                         "offset or size does not match physical rank")
            ranges = []
            for name, t in e.tensors.items():
                if not (t.dtype in ("U32", "BF16") and name and t.size > 0 and t.shape
                        and all(s > 0 for s in t.shape)
                        and (t.bits is None or 0 < t.bits <= 32)):
                    raise MoEPackFormatError(f"expert[{logical}].tensors.{name}",
                                             "invalid dtype or shape")
                end = t.offset + t.size
                if end > e.size:
                    raise MoEPackFormatError(f"expert[{logical}].tensors.{name}",
                                             "range exceeds expert blob")
                ranges.append((t.offset, end, name))
            ranges.sort()
            for a, b in zip(ranges, ranges[1:]):
                if a[1] > b[0]:
                    raise MoEPackFormatError(f"expert[{logical}].tensors",
                                             f"overlapping ranges {a[2]} and {b[2]}")


def decode_layout(data: bytes | str) -> Layout:
    """MoEPackPackedExpertsLayoutCodec.decode: JSON (the Swift Codable keys),
    then the structural validation."""
    try:
        j = json.loads(data)
        layers = []
        for lj in j["layers"]:
            experts = []
            for ej in lj["experts"]:
                tensors = {name: SubTensor(int(t["offset"]), int(t["size"]), str(t["dtype"]),
                                           [int(s) for s in t["shape"]],
                                           None if t.get("bits") is None else int(t["bits"]))
                           for name, t in ej["tensors"].items()}
                experts.append(Expert(int(ej["offset"]), int(ej["size"]), tensors,
                                      None if ej.get("expert") is None else int(ej["expert"]),
                                      None if ej.get("physicalRank") is None
                                      else int(ej["physicalRank"])))
            layers.append(Layer(int(lj["layer"]), str(lj["file"]), experts))
        layout = Layout(int(j["expertStride"]), int(j["numLayers"]), int(j["expertsPerLayer"]),
                        layers)
    except (KeyError, TypeError, ValueError, json.JSONDecodeError) as exc:
        raise MoEPackFormatError("packed_experts/layout.json", str(exc)) from None
    validate(layout)
    return layout


def encode_layout(layout: Layout) -> str:
    """MoEPackPackedExpertsLayoutCodec.encode: validated, sorted keys."""
    validate(layout)

    def sub(t: SubTensor):
        d = {"offset": t.offset, "size": t.size, "dtype": t.dtype, "shape": list(t.shape)}
        if t.bits is not None:
            d["bits"] = t.bits
        return d

    j = {"expertStride": layout.expert_stride, "numLayers": layout.num_layers,
         "expertsPerLayer": layout.experts_per_layer,
         "layers": [{"layer": lay.layer, "file": lay.file,
                     "experts": [dict({"offset": e.offset, "size": e.size,
                                       "tensors": {n: sub(t) for n, t in e.tensors.items()}},
                                      **({} if e.expert is None else {"expert": e.expert}),
                                      **({} if e.physical_rank is None
                                         else {"physicalRank": e.physical_rank}))
                                 for e in lay.experts]}
                    for lay in layout.layers]}
    return json.dumps(j, indent=2, sort_keys=True)


def read_layout(root: str | os.PathLike) -> Layout:
    return decode_layout((Path(root) / "packed_experts" / "layout.json").read_bytes())


def _role_shapes(role: str, d: int, f: int):
    return (f, d) if role in ("gate", "up") else (d, f)


def import_layer(ctx, root: str | os.PathLike, layout: Layout, layer: int, d: int, f: int):
    """One layer's expert blobs on the device in this library's layout.

    Returns the expert tensors of a MoELayer description: ``experts`` (uint8,
    ``expertsPerLayer`` blobs in logical order), ``expert_stride`` and
    ``offsets`` (tsg_expert_offsets order).  The conversion runs on the
    context's stream and is waited for: an inexact scale or a bias that is
    not -8 x scale raises ``MoEPackFormatError`` here."""
    import torch

    from .synthetic import blob_layout

    lay = next((x for x in layout.layers if x.layer == layer), None)
    if lay is None:
        raise MoEPackFormatError("layout.layers", f"no layer {layer}")
    path = Path(root) / "packed_experts" / lay.file
    raw = np.fromfile(path, dtype=np.uint8)
    if raw.size != layout.experts_per_layer * layout.expert_stride:
        raise MoEPackFormatError(f"packed_experts/{lay.file}", "wrong layer size")
    dev = torch.device("cuda", ctx.device)
    src = torch.from_numpy(raw).to(dev)
    keep = []  # staging copies alive until the conversions have run
    offsets, stride = blob_layout(d, f)
    E = layout.experts_per_layer
    out = torch.zeros(E * stride, dtype=torch.uint8, device=dev)
    torch.cuda.current_stream(dev).synchronize()  # the copies above, before the context's stream
    off = dict(zip(("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b", "down_w", "down_s",
                    "down_b"), offsets))
    for logical in range(E):
        e = layout.expert(layer, logical)
        for role in ROLES:
            rows, cols = _role_shapes(role, d, f)
            try:
                w, s = e.tensors[role], e.tensors[f"{role}_scales"]
            except KeyError as exc:
                raise MoEPackFormatError(f"expert[{logical}].tensors", f"missing {exc}") from None
            b = e.tensors.get(f"{role}_biases")
            if (w.dtype != "U32" or list(w.shape) != [rows, cols // 8] or (w.bits or 4) != 4
                    or w.size != rows * cols // 2):
                raise MoEPackFormatError(f"expert[{logical}].tensors.{role}",
                                         f"expected U32 [{rows}, {cols // 8}] int4 codes")
            if (s.dtype != "BF16" or len(s.shape) != 2 or s.shape[0] != rows
                    or cols % s.shape[1] or s.size != rows * s.shape[1] * 2):
                raise MoEPackFormatError(f"expert[{logical}].tensors.{role}_scales",
                                         "expected BF16 [rows, groups]")
            if b is not None and (b.dtype != "BF16" or list(b.shape) != list(s.shape)
                                  or b.size != s.size):
                raise MoEPackFormatError(f"expert[{logical}].tensors.{role}_biases",
                                         "expected BF16 of the scales' shape")
            group = cols // s.shape[1]
            base = src.data_ptr() + e.offset
            codes = base + w.offset
            if codes % 16:  # the device import reads 16-byte vectors
                tmp = src[e.offset + w.offset:e.offset + w.offset + w.size].clone()
                torch.cuda.current_stream(dev).synchronize()
                keep.append(tmp)
                codes = tmp.data_ptr()
            dst = out.data_ptr() + logical * stride
            check(ctx.lib.tsg_import_int4_affine(
                ctx.h, codes, base + s.offset, None if b is None else base + b.offset,
                rows, cols, group, dst + off[f"{role}_w"], dst + off[f"{role}_s"]), ctx.h)
    try:
        ctx.sync()
    except PrefillMoEGroupingError as exc:  # the device checks: an inexact scale, an affine bias
        raise MoEPackFormatError(f"packed_experts/{lay.file}", str(exc)) from None
    del keep, src
    return {"experts": out, "expert_stride": stride, "offsets": offsets}


__all__ = ["ALIGNMENT", "MoEPackFormatError", "SubTensor", "Expert", "Layer", "Layout",
           "validate", "decode_layout", "encode_layout", "read_layout", "import_layer"]
