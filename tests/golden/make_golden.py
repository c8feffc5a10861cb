"""Generate tests/golden/ref_golden.npz from the reference's own CPU code.

The reference's CPU model functions (engine/src/gguf_loader.cpp, compiled
unchanged by oracle/Makefile into oracle/_ref/libiq36_ref.so) are run on small
seeded inputs; their outputs pin the CPU restatement in oracle/ (checked by
tests/test_oracle_golden.py, which needs neither the reference checkout nor a
GPU). Run from the repository root:

    make -C oracle ref && python tests/golden/make_golden.py
"""

from __future__ import annotations

import ctypes
import sys
from ctypes import c_float, c_int, c_void_p
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle  # noqa: E402


def p(a):
    return a.ctypes.data_as(c_void_p)


def main() -> None:
    ref = oracle.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libiq36_ref.so missing: run `make -C oracle ref` first")
    rng = np.random.default_rng(20260627)
    out: dict[str, np.ndarray] = {}

    # --- router selection (select_router_topk, gguf_loader.cpp:3733-3743) ---
    cases = []
    cases.append(rng.standard_normal(256).astype(np.float32))
    tie = rng.standard_normal(256).astype(np.float32)
    top = np.argsort(-tie)
    tie[top[6]] = tie[top[7]] = tie[top[8]] = tie[top[9]]  # ties across the k boundary
    tie[200] = tie[top[0]]                                  # tie at rank 0
    cases.append(tie)
    cases.append((rng.standard_normal(256) * 8 - 40).astype(np.float32))
    cases.append(np.zeros(256, np.float32))                 # all equal
    router_logits = np.stack(cases)
    ids = np.zeros((len(cases), 8), np.int32)
    probs = np.zeros((len(cases), 8), np.float32)
    norm = np.zeros((len(cases), 8), np.float32)
    for i, lg in enumerate(router_logits):
        lg = np.ascontiguousarray(lg)
        ref.ref_router_select(p(lg), c_int(256), c_int(8), c_float(6.103515625e-5),
                              p(ids[i]), p(probs[i]), p(norm[i]))
    out.update(router_logits=router_logits, router_ids=ids, router_probs=probs,
               router_norm=norm)

    # --- SwiGLU from gate_up (:4640-4668) ---
    gu = (rng.standard_normal((2, 2 * 64)) * 3).astype(np.float32)
    sw = np.zeros(2 * 64, np.float32)
    ref.ref_swiglu_from_gate_up(p(gu), c_int(64), c_int(2), p(sw))
    out.update(swiglu_gate_up=gu, swiglu_out=sw)

    # --- expert weights + aggregate (:3773-3819) ---
    dn = rng.standard_normal((3, 64)).astype(np.float32)
    w = np.array([0.5, 0.3, 0.2], np.float32)
    agg = np.zeros(64, np.float32)
    ref.ref_weight_aggregate(p(dn), p(w), c_int(3), c_int(64), p(agg))
    out.update(agg_down=dn, agg_weights=w, agg_out=agg)

    # --- RMSNorm (:3368-3391) and repeated RMSNorm (:3410-3439) ---
    x = (rng.standard_normal(2048) * 4).astype(np.float32)
    nw = rng.uniform(0.9, 1.1, 2048).astype(np.float32)
    rn = np.zeros(2048, np.float32)
    ref.ref_rms_norm(p(x), c_int(2048), p(nw), c_int(2048), c_float(1e-6), p(rn))
    xr = (rng.standard_normal(16 * 256) * 2).astype(np.float32)
    nwr = rng.uniform(0.9, 1.1, 256).astype(np.float32)
    rr = np.zeros(16 * 256, np.float32)
    ref.ref_rms_norm(p(xr), c_int(16 * 256), p(nwr), c_int(256), c_float(1e-6), p(rr))
    out.update(rms_x=x, rms_w=nw, rms_out=rn, rrms_x=xr, rrms_w=nwr, rrms_out=rr)

    # --- attention core (:6071-6137) + gate (:6034-6069), fp16-valued inputs ---
    T = 37
    q = rng.standard_normal(16 * 256).astype(np.float16).astype(np.float32)
    kh = rng.standard_normal((T, 2 * 256)).astype(np.float16).astype(np.float32)
    vh = rng.standard_normal((T, 2 * 256)).astype(np.float16).astype(np.float32)
    pre = np.zeros(16 * 256, np.float32)
    ref.ref_attention_core(p(q), p(kh), p(vh), c_int(T), c_int(256), c_int(16), c_int(2),
                           c_float(1.0 / 16.0), p(pre))
    qf = rng.standard_normal(16 * 2 * 256).astype(np.float16).astype(np.float32)
    gated = np.zeros(16 * 256, np.float32)
    ref.ref_attention_gate(p(qf), p(pre), c_int(16), c_int(256), p(gated))
    out.update(attn_q=q, attn_k=kh, attn_v=vh, attn_pregate=pre, attn_qfull=qf,
               attn_gated=gated)

    # --- DeltaNet delta core (:4670-4788), one query head per value head ---
    D, nv, nk = 128, 4, 2
    act = rng.standard_normal((2 * nk + nv) * D).astype(np.float16).astype(np.float32)
    g = -rng.uniform(0.05, 1.0, nv).astype(np.float32)
    beta = rng.uniform(0.1, 0.9, nv).astype(np.float32)
    state = (rng.standard_normal((nv, D, D)) * 0.1).astype(np.float32)  # [v][key][value]
    z = rng.standard_normal(nv * D).astype(np.float16).astype(np.float32)
    dnw = rng.uniform(0.9, 1.1, D).astype(np.float32)
    final = np.zeros(nv * D, np.float32)
    new_state = np.zeros((nv, D, D), np.float32)
    for vh_ in range(nv):
        kh_ = vh_ // (nv // nk)  # OpenVINO head mapping (iq36_gated_delta_net.cl:46)
        qv = act[kh_ * D:(kh_ + 1) * D].astype(np.float64)
        kv = act[(nk + kh_) * D:(nk + kh_ + 1) * D].astype(np.float64)
        qn = (qv / np.sqrt((qv * qv).sum() + 1e-6)).astype(np.float32)
        kn = (kv / np.sqrt((kv * kv).sum() + 1e-6)).astype(np.float32)
        vv = np.ascontiguousarray(act[(2 * nk + vh_) * D:(2 * nk + vh_ + 1) * D])
        st = np.ascontiguousarray(state[vh_].T)  # reference layout [value row][key col]
        a_o = np.zeros(D, np.float32)
        s_o = np.zeros((D, D), np.float32)
        f_o = np.zeros(D, np.float32)
        gg = np.ascontiguousarray(g[vh_:vh_ + 1])
        bb = np.ascontiguousarray(beta[vh_:vh_ + 1])
        zz = np.ascontiguousarray(z[vh_ * D:(vh_ + 1) * D])
        ref.ref_delta_core(p(qn), p(kn), p(vv), p(gg), p(bb), p(st), p(zz), p(dnw), c_int(1),
                           c_int(1), c_int(D), c_float(1e-6), p(a_o), p(s_o), p(f_o))
        final[vh_ * D:(vh_ + 1) * D] = f_o
        new_state[vh_] = s_o.T
    out.update(delta_act=act, delta_g=g, delta_beta=beta, delta_state=state, delta_z=z,
               delta_norm_w=dnw, delta_final=final, delta_new_state=new_state,
               delta_dims=np.array([D, nv, nk], np.int32))

    # --- sigmoid_scalar (:3638-3644) ---
    sx = np.array([-30.0, -5.0, -0.5, 0.0, 0.25, 3.0, 40.0], np.float32)
    out.update(sigmoid_x=sx, sigmoid_y=np.array([ref.ref_sigmoid_scalar(float(v)) for v in sx],
                                                np.float32))

    path = Path(__file__).with_name("ref_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
