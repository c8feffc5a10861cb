"""Generate tests/golden/group_major_golden.npz from the reference's own repack code.

The reference's fixed-FC graph rewrite (tools/intel_qwen36_openvino_fixed_fc.py,
`_packed_weight`, `_group_major_scale`, `_group_major_zero_point`, :218-258)
turns the OpenVINO compressed constants of a u4 projection (weight u4
[M, groups, G], scale f16 [M, groups, 1], zero point u4 [M, groups, 1], each
packed two nibbles per byte, low nibble first) into the inputs of its custom
FC op: the weight bytes unchanged, the scales and zero points transposed to
group-major order. The module imports only the standard library (OpenVINO and
numpy are passed in), so it runs here with numpy and a small stand-in for the
two OpenVINO calls it makes (`opset13.constant` and `Type`). The fixture pins
the adapter in `engine/ov_ir.py` and `iq36_u4_layout_from_group_major`.
Run from the repository root with the reference checked out at REF:

    python tests/golden/make_group_major_golden.py REF
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1].parent


class _Const:
    """Stand-in for an OpenVINO Constant: holds data and a friendly name."""

    def __init__(self, data, name="c"):
        self.data = np.asarray(data)
        self.name = name

    def get_data(self):
        return self.data

    def get_friendly_name(self):
        return self.name

    def set_friendly_name(self, name):
        self.name = name


class _Opset:
    @staticmethod
    def constant(values, dtype=None):
        return _Const(np.array(values, copy=True))


class _Type:
    f16 = "f16"
    u8 = "u8"
    u4 = "u4"


class _Ov:
    opset13 = _Opset()
    Type = _Type()


def pack_u4(q: np.ndarray) -> np.ndarray:
    q = q.reshape(-1)
    return (q[0::2] & 15 | (q[1::2] & 15) << 4).astype(np.uint8)


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else "../reference")
    sys.path.insert(0, str(ref / "tools"))
    import intel_qwen36_openvino_fixed_fc as ffc  # the reference module

    rng = np.random.default_rng(20261202)
    out = {}
    for name, m, k, g in (("g64", 96, 512, 64), ("g128", 40, 1024, 128)):
        groups = k // g
        q = rng.integers(0, 16, size=(m, groups, g), dtype=np.uint8)
        zp = rng.integers(0, 16, size=(m, groups, 1), dtype=np.uint8)
        sc = rng.uniform(0.005, 0.02, size=(m, groups, 1)).astype(np.float16)
        proj = {"weight": _Const(pack_u4(q)), "scale": _Const(sc),
                "zero_point": _Const(pack_u4(zp)), "m": m, "groups": groups}
        w_gm = ffc._packed_weight(_Ov, np, proj).get_data().reshape(-1)
        s_gm = ffc._group_major_scale(_Ov, np, proj).get_data().reshape(-1)
        z_gm = ffc._group_major_zero_point(_Ov, np, proj).get_data().reshape(-1)
        out[f"{name}_dims"] = np.array([m, k, g], np.int32)
        out[f"{name}_weight"] = pack_u4(q)            # OV row-major [M, K/2]
        out[f"{name}_scale"] = sc.reshape(m, groups)  # OV row-major [M, groups]
        out[f"{name}_zp"] = pack_u4(zp)               # OV row-major [M*groups/2]
        out[f"{name}_weight_gm"] = w_gm
        out[f"{name}_scale_gm"] = s_gm
        out[f"{name}_zp_gm"] = z_gm
    dst = ROOT / "tests" / "golden" / "group_major_golden.npz"
    np.savez_compressed(dst, **out)
    print("wrote", dst, sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main()
