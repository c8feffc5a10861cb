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


def test_u4_row_ranges_and_k_slices_dequantise_to_the_slices():
    """The tensor-parallel slicing helpers: gathered row ranges and K slices of
    a u4 matrix dequantise to the same rows / columns of the full matrix
    (zero-point nibbles repacked exactly)."""
    import numpy as np
    import torch
    from engine.tp_decode import u4_cols, u4_rows
    from engine.ops import U4Weight
    from helpers import dequant_u4, make_u4
    rng = np.random.default_rng(3)
    w, s, z = make_u4(rng, 96, 1024)
    full = dequant_u4(w, s, z)
    t = U4Weight(torch.from_numpy(w), torch.from_numpy(s), torch.from_numpy(z), 128)
    ranges = [(0, 16), (48, 64), (80, 96)]
    r = u4_rows(t, ranges)
    got = dequant_u4(r.weight.numpy(), r.scale.numpy(), r.zp.numpy())
    want = np.concatenate([full[a:b] for a, b in ranges])
    np.testing.assert_array_equal(got, want)
    c = u4_cols(t, 256, 768)
    got = dequant_u4(c.weight.numpy(), c.scale.numpy(), c.zp.numpy())
    np.testing.assert_array_equal(got, full[:, 256:768])
