"""The decode step's kernels compile without register spills (CPU; nvcc only).

A spill in a decode-path kernel costs on every launch of every step: a
chunk-list branch added to the weight-stream GEMV once made its only
instantiation spill 24 bytes and slowed the decode step by ~4%, with every
numerical test still green. This test compiles the decode-path sources for
sm_100a with `-Xptxas -v` and checks the ptxas report of each kernel the
decode graph launches.
"""

import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "aima-intel-plk-qwen36-35b-u4-engine_b200"

# source file -> kernels of the decode step (substrings of the mangled names)
DECODE_KERNELS = {
    "u4_stream.cu": ["u4_stream_proj_kernelILi128ELb0E"],
    "moe_decode.cu": ["moe_layer_kernel"],
    "model_ops.cu": ["delta_step_kernel", "delta_prep_kernel", "attn_prep_kernel",
                     "argmax_partial_kernel", "argmax_final_kernel", "embed_kernel",
                     "decode_positions_kernel"],
    "paged_gqa.cu": ["gqa_split_kernel", "gqa_combine_kernel"],
}


def _ptxas_report(src: Path) -> dict[str, str]:
    sys.path.insert(0, str(PKG))
    import build as B
    r = subprocess.run([B.nvcc(), *B.NVCC_FLAGS, "-Xptxas", "-v", "-c", str(src), "-o",
                        "/dev/null"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    out: dict[str, str] = {}
    name = None
    for line in r.stderr.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            name = m.group(1)
        elif name and "spill stores" in line:
            out[name] = line
            name = None
    return out


@pytest.mark.parametrize("src", sorted(DECODE_KERNELS))
def test_decode_kernels_do_not_spill(src):
    report = _ptxas_report(PKG / "csrc" / src)
    for kernel in DECODE_KERNELS[src]:
        hits = {n: l for n, l in report.items() if kernel in n}
        assert hits, f"{kernel} not found in the ptxas report of {src}"
        for n, line in hits.items():
            m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
            assert m, line
            assert m.group(1) == "0" and m.group(2) == "0", f"{n}: {line.strip()}"
