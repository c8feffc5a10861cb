"""B200 (sm_100a) batch-1 hot path of a Qwen3.6-35B-A3B-shaped hybrid MoE.

``engine.ops`` is the operator boundary (u4 GEMV, router top-k, MoE expert
FFN decode/prefill, paged GQA decode); ``engine.runtime`` is the host decode
loop of the synthetic config-4 model; ``engine.parallel_ep`` and
``engine.parallel_tp`` hold the multi-GPU expert- and tensor-parallel paths.
"""

from . import _native  # noqa: F401

__all__ = ["_native"]
