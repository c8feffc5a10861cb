"""Row sharding inside the experts (tensor-parallel MoE decode) on the CPU:
the oracle's MoE block over each rank's shard, summed over ranks, equals the
unsharded block (fp32 summation order aside)."""

import numpy as np
import torch

from helpers import make_bank
from oracle import oracle


def _np_bank(b):
    return {"gu_w": b.gate_up_weight.numpy(), "gu_s": b.gate_up_scale.numpy(),
            "gu_z": b.gate_up_zp.numpy(), "d_w": b.down_weight.numpy(),
            "d_s": b.down_scale.numpy(), "d_z": b.down_zp.numpy()}


def test_row_shards_sum_to_the_block():
    from engine.ops import ExpertBank
    from engine.parallel_tp import shard_expert_bank_rows
    rng = np.random.default_rng(3)
    E, H, I, k = 8, 256, 512, 4
    bank = make_bank(rng, E, H, I)
    shared = make_bank(rng, 1, H, I)
    tb = ExpertBank(*(torch.from_numpy(np.ascontiguousarray(bank[n])) for n in
                      ("gu_w", "gu_s", "gu_z", "d_w", "d_s", "d_z")), 128)
    ts = ExpertBank(*(torch.from_numpy(np.ascontiguousarray(shared[n])) for n in
                      ("gu_w", "gu_s", "gu_z", "d_w", "d_s", "d_z")), 128)
    x = rng.standard_normal(H).astype(np.float16)
    ids = np.array([5, 1, 7, 2], np.int32)
    w = np.array([0.4, 0.3, 0.2, 0.1], np.float32)
    sl = 0.25
    ref = oracle.moe_decode(x, ids, w, bank, {kk: v[0] for kk, v in shared.items()}, sl, 128)
    for world in (2, 4):
        tot = np.zeros(H, np.float64)
        for r in range(world):
            b = _np_bank(shard_expert_bank_rows(tb, r, world))
            s = {kk: v[0] for kk, v in _np_bank(shard_expert_bank_rows(ts, r, world)).items()}
            assert b["gu_w"].shape == (E, 2 * I // world, H // 2)
            assert b["d_w"].shape == (E, H, I // world // 2)
            tot += oracle.moe_decode(x, ids, w, b, s, sl, 128)
        err = np.max(np.abs(tot - ref)) / np.max(np.abs(ref))
        assert err < 1e-5, (world, err)
