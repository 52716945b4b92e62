"""CPU checks of the host-side weight layouts the fused kernels take."""
import numpy as np
import torch

import oracle
from anvilq_b200 import ops, synthetic


def test_mlp_interleave_moves_whole_words():
    """gate|up in unit-interleaved order: word 8u + w is gate word 4u + w, word
    8u + 4 + w is up word 4u + w; scales and zeros move with their columns."""
    H, I = 256, 96
    rng = np.random.default_rng(3)
    qw = torch.from_numpy(rng.integers(0, 2**31, (H, 2 * I // 8), dtype=np.int64).astype(np.int32))
    qz = torch.from_numpy(rng.integers(0, 2**31, (H // 128, 2 * I // 8), dtype=np.int64).astype(np.int32))
    sc = torch.from_numpy(rng.standard_normal((H // 128, 2 * I)).astype(np.float16))
    iq, iz, isc = ops.mlp_interleave(qw, qz, sc)
    gw, uw = qw[:, :I // 8], qw[:, I // 8:]
    for u in range(I // 32):
        for w in range(4):
            assert torch.equal(iq[:, 8 * u + w], gw[:, 4 * u + w])
            assert torch.equal(iq[:, 8 * u + 4 + w], uw[:, 4 * u + w])
            assert torch.equal(iz[:, 8 * u + w], qz[:, 4 * u + w])
            assert torch.equal(iz[:, 8 * u + 4 + w], qz[:, I // 8 + 4 * u + w])
        assert torch.equal(isc[:, 64 * u:64 * u + 32], sc[:, 32 * u:32 * u + 32])
        assert torch.equal(isc[:, 64 * u + 32:64 * u + 64], sc[:, I + 32 * u:I + 32 * u + 32])


def test_mlp_interleave_keeps_the_projection():
    """The interleaved weights give the same gate and up outputs, column for
    column, as the concatenated ones (the oracle GEMV on both)."""
    H, I = 256, 64
    x, layer = synthetic.gemv_case(1, H, 2 * I, 128, seed=5)
    iq, iz, isc = ops.mlp_interleave(torch.from_numpy(layer.qweight), torch.from_numpy(layer.qzeros),
                                     torch.from_numpy(layer.scales))
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits, None, 128)[0]
    got = oracle.gemv_fp32(x.astype(np.float32), iq.numpy(), iz.numpy(), isc.numpy().view(np.uint16), None,
                           128)[0]
    g_ref, u_ref = ref[:I], ref[I:]
    for u in range(I // 32):
        assert np.array_equal(got[64 * u:64 * u + 32], g_ref[32 * u:32 * u + 32])
        assert np.array_equal(got[64 * u + 32:64 * u + 64], u_ref[32 * u:32 * u + 32])
