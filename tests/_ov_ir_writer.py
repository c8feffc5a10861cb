"""Test helper: write a small OpenVINO IR (xml + bin) holding compressed u4
projections in the subgraph form the reference traces
(tools/intel_qwen36_openvino_fixed_fc.py:107-145). Test infrastructure only."""

from __future__ import annotations

from pathlib import Path

import numpy as np


def write_ir(path: Path, projections: list[dict]) -> None:
    """projections: dicts with name, m, k, group, weight [M, K/2] u8 packed,
    scale [M, groups] f16, zp [M*groups/2] u8 packed."""
    layers, edges, blob = [], [], bytearray()
    nid = [0]

    def layer(kind, name, data=None, n_in=0):
        lid = nid[0]
        nid[0] += 1
        attrs = "".join(f' {k}="{v}"' for k, v in (data or {}).items())
        ports_in = "".join(f'<port id="{i}"/>' for i in range(n_in))
        layers.append(f'<layer id="{lid}" name="{name}" type="{kind}" version="opset1">'
                      f'<data{attrs}/>' + (f"<input>{ports_in}</input>" if n_in else "") +
                      f'<output><port id="{n_in}"/></output></layer>')
        return lid, n_in

    def edge(src, dst, port):
        edges.append(f'<edge from-layer="{src[0]}" from-port="{src[1]}" to-layer="{dst[0]}" '
                     f'to-port="{port}"/>')

    def const(name, arr, et, shape):
        off = len(blob)
        blob.extend(np.ascontiguousarray(arr).tobytes())
        return layer("Const", name, {"element_type": et, "shape": ",".join(map(str, shape)),
                                     "offset": off, "size": len(blob) - off})

    x = layer("Parameter", "x", {"shape": "1,1", "element_type": "f32"})
    for p in projections:
        m, k, g = p["m"], p["k"], p["group"]
        groups = k // g
        w = const(p["name"] + "/w", p["weight"], "u4", [m, groups, g])
        z = const(p["name"] + "/zp", p["zp"], "u4", [m, groups, 1])
        s = const(p["name"] + "/scale", p["scale"], "f16", [m, groups, 1])
        cw = layer("Convert", p["name"] + "/cw", {"destination_type": "f16"}, 1)
        edge(w, cw, 0)
        cz = layer("Convert", p["name"] + "/cz", {"destination_type": "f16"}, 1)
        edge(z, cz, 0)
        sub = layer("Subtract", p["name"] + "/sub", {}, 2)
        edge(cw, sub, 0)
        edge(cz, sub, 1)
        mul = layer("Multiply", p["name"] + "/mul", {}, 2)
        edge(sub, mul, 0)
        edge(s, mul, 1)
        shp = const(p["name"] + "/shape", np.array([m, k], np.int64), "i64", [2])
        rsh = layer("Reshape", p["name"] + "/reshape", {"special_zero": "false"}, 2)
        edge(mul, rsh, 0)
        edge(shp, rsh, 1)
        cf = layer("Convert", p["name"] + "/cf", {"destination_type": "f32"}, 1)
        edge(rsh, cf, 0)
        mm = layer("MatMul", p["name"], {"transpose_a": "false", "transpose_b": "true"}, 2)
        edge(x, mm, 0)
        edge(cf, mm, 1)
    xml = ('<?xml version="1.0"?>\n<net name="t" version="11"><layers>' + "".join(layers) +
           "</layers><edges>" + "".join(edges) + "</edges></net>\n")
    path.with_suffix(".xml").write_text(xml)
    path.with_suffix(".bin").write_bytes(bytes(blob))
