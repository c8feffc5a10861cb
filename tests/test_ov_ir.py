"""On-disk format adapter (engine/ov_ir.py) and the group-major layout map.

CPU: the reference's own fixed-FC repack (tools/intel_qwen36_openvino_fixed_fc.py
:218-258, run by tests/golden/make_group_major_golden.py) pins a numpy
restatement of its inverse; an IR written by tests/_ov_ir_writer.py in the
reference's compressed-projection form reads back to the same constants. GPU:
iq36_u4_layout_from_group_major / to_group_major reproduce the fixture bit for
bit, and a projection loaded from the IR gives the oracle's GEMV.
"""

from pathlib import Path

import numpy as np
import pytest

from _ov_ir_writer import write_ir
from oracle import oracle

G = np.load(Path(__file__).parent / "golden" / "group_major_golden.npz")
CASES = ("g64", "g128")


def _unpack(b):
    out = np.empty(b.size * 2, np.uint8)
    out[0::2], out[1::2] = b & 15, b >> 4
    return out


def _pack(q):
    return (q[0::2] & 15 | (q[1::2] & 15) << 4).astype(np.uint8)


def _from_group_major(scale_gm, zp_gm, m, groups):
    scale = scale_gm.reshape(groups, m).T.copy()
    zp = _pack(_unpack(zp_gm)[:m * groups].reshape(groups, m).T.reshape(-1))
    return scale, zp


@pytest.mark.parametrize("case", CASES)
def test_group_major_inverse_matches_reference_repack(case):
    m, k, g = (int(v) for v in G[f"{case}_dims"])
    scale, zp = _from_group_major(G[f"{case}_scale_gm"], G[f"{case}_zp_gm"], m, k // g)
    np.testing.assert_array_equal(scale, G[f"{case}_scale"])
    np.testing.assert_array_equal(zp, G[f"{case}_zp"])
    np.testing.assert_array_equal(G[f"{case}_weight_gm"], G[f"{case}_weight"])  # bytes kept


def _projections():
    out = []
    for case in CASES:
        m, k, g = (int(v) for v in G[f"{case}_dims"])
        out.append({"name": f"proj_{case}", "m": m, "k": k, "group": g,
                    "weight": G[f"{case}_weight"].reshape(m, k // 2),
                    "scale": G[f"{case}_scale"], "zp": G[f"{case}_zp"]})
    return out


def test_ir_reader_returns_the_compressed_constants(tmp_path):
    from engine import ov_ir
    projs = _projections()
    write_ir(tmp_path / "model", projs)
    ir = ov_ir.read_ir(tmp_path / "model.xml")
    got = {p["name"]: p for p in ov_ir.compressed_projections(ir)}
    assert sorted(got) == sorted(p["name"] for p in projs)
    for p in projs:
        q = got[p["name"]]
        assert (q["m"], q["k"], q["group"]) == (p["m"], p["k"], p["group"])
        np.testing.assert_array_equal(q["weight"], p["weight"])
        np.testing.assert_array_equal(q["scale"].view(np.float16), p["scale"])
        np.testing.assert_array_equal(q["zp"], p["zp"])


def test_ir_reader_rejects_a_non_u4_weight(tmp_path):
    from engine import ov_ir
    p = _projections()[0]
    write_ir(tmp_path / "m", [p])
    xml = (tmp_path / "m.xml").read_text().replace('element_type="u4" shape="96,8,64"',
                                                   'element_type="u8" shape="96,8,64"', 1)
    (tmp_path / "m.xml").write_text(xml)
    with pytest.raises(ValueError):
        ir = ov_ir.read_ir(tmp_path / "m.xml")
        ov_ir.trace_projection(ir, next(l for l in ir.layers.values() if l.type == "MatMul"))


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_layout_adapter_kernels_match_reference_repack(cuda, case):
    import torch
    from engine import _native as N
    from engine.ops import _stream
    m, k, g = (int(v) for v in G[f"{case}_dims"])
    groups = k // g
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    s_out = torch.empty(m, groups, dtype=torch.float16, device=cuda)
    z_out = torch.empty(m * groups // 2, dtype=torch.uint8, device=cuda)
    s_in, z_in = t(G[f"{case}_scale_gm"]), t(G[f"{case}_zp_gm"])  # held across the launch
    N.call("iq36_u4_layout_from_group_major", s_in.data_ptr(), z_in.data_ptr(), m, groups,
           s_out.data_ptr(), z_out.data_ptr(), _stream(cuda))
    np.testing.assert_array_equal(s_out.cpu().numpy(), G[f"{case}_scale"])
    np.testing.assert_array_equal(z_out.cpu().numpy(), G[f"{case}_zp"])
    s_gm = torch.empty(groups * m, dtype=torch.float16, device=cuda)
    z_gm = torch.empty_like(z_out)
    N.call("iq36_u4_layout_to_group_major", s_out.data_ptr(), z_out.data_ptr(), m, groups,
           s_gm.data_ptr(), z_gm.data_ptr(), _stream(cuda))
    np.testing.assert_array_equal(s_gm.cpu().numpy(), G[f"{case}_scale_gm"])
    np.testing.assert_array_equal(z_gm.cpu().numpy(), G[f"{case}_zp_gm"])


@pytest.mark.gpu
def test_projection_loaded_from_ir_runs_the_gemv(cuda, tmp_path):
    import torch
    from engine import ov_ir
    from engine.ops import u4_matvec
    write_ir(tmp_path / "model", _projections())
    ir = ov_ir.read_ir(tmp_path / "model.xml")
    for p in ov_ir.compressed_projections(ir):
        w = ov_ir.load_projection(p, cuda)
        x = np.random.default_rng(p["m"]).standard_normal(p["k"]).astype(np.float16)
        out = u4_matvec(torch.from_numpy(x).to(cuda), w, out_dtype=torch.float32)
        ref = oracle.u4_gemv(x, p["weight"], p["scale"].view(np.float16), p["zp"], p["group"])
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-3,
                                   atol=2e-3 * float(np.abs(ref).max()))
        # and the fixed-FC input form maps back to the same matrix
        s_gm = torch.from_numpy(np.ascontiguousarray(p["scale"].view(np.float16).T)).to(cuda)
        qz = _unpack(p["zp"]).reshape(p["m"], -1).T.reshape(-1)
        z_gm = torch.from_numpy(_pack(qz)).to(cuda)
        w2 = ov_ir.u4_from_group_major(torch.from_numpy(p["weight"]).to(cuda), s_gm, z_gm,
                                       p["m"], p["k"], p["group"])
        assert torch.equal(w2.scale, w.scale) and torch.equal(w2.zp, w.zp)
