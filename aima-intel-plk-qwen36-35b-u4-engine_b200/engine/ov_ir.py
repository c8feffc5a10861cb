"""On-disk format adapter: OpenVINO u4 IR weights into the kernels' u4 layout.

The reference's checkpoint is an OpenVINO IR (an ``.xml`` graph and a ``.bin``
blob). Each compressed projection is the subgraph the reference traces in
``trace_compressed_projection`` (tools/intel_qwen36_openvino_fixed_fc.py:107-145):

    MatMul(activation, Convert(Reshape(Multiply(Subtract(Convert(W u4),
                                                         Convert(ZP u4)),
                                                SCALE f16))))

with W u4 [M, groups, G], ZP u4 [M, groups, 1], SCALE f16 [M, groups, 1], u4
packed two per byte, low nibble first. That is exactly the row-major layout
the kernels here read (include/iq36_b200.h), so loading is a byte copy of the
three constants. The reference's own fixed-FC op instead feeds group-major
scales and zero points (fixed_fc.py:218-258); ``u4_from_group_major`` maps
that form back (``iq36_u4_layout_from_group_major``) for a host that holds the
repacked tensors.

``read_ir`` parses the IR's layers and edges (no OpenVINO needed);
``compressed_projections`` finds the subgraphs above and returns their
constants as numpy arrays; ``load_projection`` puts one on the device as a
``U4Weight``.
"""

from __future__ import annotations

import xml.etree.ElementTree as ET
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

_DTYPES = {"f16": (np.float16, 16), "f32": (np.float32, 32), "u8": (np.uint8, 8),
           "i32": (np.int32, 32), "i64": (np.int64, 64), "u4": (np.uint8, 4)}


@dataclass
class Layer:
    id: str
    name: str
    type: str
    data: dict
    inputs: list = field(default_factory=list)  # producer layer ids, by input port order


@dataclass
class IR:
    layers: dict  # id -> Layer
    blob: bytes

    def const(self, layer: Layer) -> np.ndarray:
        """A Const layer's data: u4 stays packed (one byte holds two elements)."""
        et = layer.data["element_type"]
        if et not in _DTYPES:
            raise ValueError(f"{layer.name}: unsupported constant type {et}")
        off, size = int(layer.data["offset"]), int(layer.data["size"])
        if off < 0 or off + size > len(self.blob):
            raise ValueError(f"{layer.name}: constant lies outside the blob")
        dt, bits = _DTYPES[et]
        shape = _shape(layer.data.get("shape", ""))
        count = int(np.prod(shape)) if shape else 1
        if size * 8 != count * bits:
            raise ValueError(f"{layer.name}: size {size} does not hold {count} x {et}")
        return np.frombuffer(self.blob, dtype=dt, count=size * 8 // max(bits, 8),
                             offset=off).copy()


def _shape(text: str) -> list[int]:
    text = text.strip()
    return [int(v) for v in text.split(",")] if text else []


def read_ir(xml_path: str | Path, bin_path: str | Path | None = None) -> IR:
    xml_path = Path(xml_path)
    bin_path = Path(bin_path) if bin_path else xml_path.with_suffix(".bin")
    root = ET.parse(xml_path).getroot()
    layers = {}
    for el in root.find("layers"):
        d = el.find("data")
        layers[el.get("id")] = Layer(el.get("id"), el.get("name"), el.get("type"),
                                     dict(d.attrib) if d is not None else {})
    ins: dict[str, list[tuple[int, str]]] = {}
    for e in root.find("edges"):
        ins.setdefault(e.get("to-layer"), []).append((int(e.get("to-port")), e.get("from-layer")))
    for lid, lst in ins.items():
        layers[lid].inputs = [src for _, src in sorted(lst)]
    return IR(layers, bin_path.read_bytes())


def _expect(ir: IR, lid: str, kind: str, ctx: str) -> Layer:
    layer = ir.layers[lid]
    if layer.type != kind:
        raise ValueError(f"{ctx}: expected {kind}, found {layer.type} at {layer.name}")
    return layer


def trace_projection(ir: IR, matmul: Layer) -> dict:
    """The compressed constants of one MatMul (the reference's trace,
    fixed_fc.py:107-145), as numpy arrays in the kernels' layout."""
    ctx = matmul.name
    cvt = _expect(ir, matmul.inputs[1], "Convert", ctx)
    rsh = _expect(ir, cvt.inputs[0], "Reshape", ctx)
    mul = _expect(ir, rsh.inputs[0], "Multiply", ctx)
    sub = _expect(ir, mul.inputs[0], "Subtract", ctx)
    wc = _expect(ir, _expect(ir, sub.inputs[0], "Convert", ctx).inputs[0], "Const", ctx)
    zc = _expect(ir, _expect(ir, sub.inputs[1], "Convert", ctx).inputs[0], "Const", ctx)
    sc = _expect(ir, mul.inputs[1], "Const", ctx)
    if wc.data.get("element_type") != "u4" or zc.data.get("element_type") != "u4":
        raise ValueError(f"{ctx}: weight or zero point is not u4")
    if sc.data.get("element_type") != "f16":
        raise ValueError(f"{ctx}: scale is not f16")
    shape = _shape(wc.data["shape"])
    if len(shape) != 3:
        raise ValueError(f"{ctx}: packed weight shape {shape} is not [M, groups, G]")
    m, groups, g = shape
    if _shape(zc.data["shape"]) != [m, groups, 1] or _shape(sc.data["shape"]) != [m, groups, 1]:
        raise ValueError(f"{ctx}: scale / zero-point shape is not [M, groups, 1]")
    if (m * groups) % 2:
        raise ValueError(f"{ctx}: zero points of an odd element count")
    return {"name": ctx, "m": m, "k": groups * g, "group": g,
            "weight": ir.const(wc).reshape(m, groups * g // 2),
            "scale": ir.const(sc).reshape(m, groups),
            "zp": ir.const(zc)}


def compressed_projections(ir: IR) -> list[dict]:
    """Every MatMul fed by the compressed-weight subgraph, in layer order."""
    out = []
    for layer in ir.layers.values():
        if layer.type == "MatMul" and len(layer.inputs) == 2:
            try:
                out.append(trace_projection(ir, layer))
            except (ValueError, KeyError, IndexError):
                continue
    return out


def load_projection(p: dict, device):
    """numpy constants of one projection -> device ``U4Weight``."""
    import torch

    from . import ops
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
    w = ops.U4Weight(t(p["weight"]), t(p["scale"].view(np.float16)), t(p["zp"]), p["group"])
    w.validate()
    return w


def u4_from_group_major(weight_packed, scale_gm, zp_gm, rows: int, k: int, group: int):
    """Device tensors in the reference's fixed-FC input form (weight bytes,
    group-major scale [groups, rows] fp16 and zero points) -> ``U4Weight``."""
    import torch

    from . import _native as N
    from . import ops
    groups = k // group
    dev = weight_packed.device
    scale = torch.empty(rows, groups, dtype=torch.float16, device=dev)
    zp = torch.empty(rows * groups // 2, dtype=torch.uint8, device=dev)
    N.call("iq36_u4_layout_from_group_major", scale_gm.data_ptr(), zp_gm.data_ptr(), rows,
           groups, scale.data_ptr(), zp.data_ptr(), ops._stream(dev))
    w = ops.U4Weight(weight_packed.reshape(rows, k // 2), scale, zp, group)
    w.validate()
    return w
