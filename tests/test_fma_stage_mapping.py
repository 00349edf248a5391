"""Index arithmetic of the CUDA-core consumer stage (``fma_stage`` in
``csrc/pkv_kernels.cuh``), restated with numpy over 32 simulated lanes: the
reduce-scatter leaves lane l the warp-wide sums of values 2l and 2l + 1
(token l >> 1, heads 2 (l & 1) and 2 (l & 1) + 1); the probability
broadcast reads token t's heads from lanes 2t and 2t + 1; lane l's 4 dims
are one 8-byte part of 16-byte chunk (l >> 1) & 7 of half-row l >> 4."""

import numpy as np


def reduce_scatter(part):
    """part: [32 lanes][64 values] -> [32][2] as the kernel's 5 xor levels."""
    v = part.copy()
    n = 64
    for lvl in range(5):
        off, half = 16 >> lvl, 32 >> lvl
        nxt = np.empty((32, half))
        for lane in range(32):
            upper = (lane & off) != 0
            send_peer = v[lane ^ off]
            for i in range(half):
                keep = v[lane, i + half] if upper else v[lane, i]
                # the peer sends the half this lane keeps
                recv = send_peer[i + half] if upper else send_peer[i]
                nxt[lane, i] = keep + recv
        v = nxt
        n //= 2
    assert n == 2
    return v


def test_reduce_scatter_leaves_lane_l_values_2l_and_2l_plus_1():
    rng = np.random.default_rng(0)
    part = rng.standard_normal((32, 64))
    got = reduce_scatter(part)
    total = part.sum(axis=0)
    for lane in range(32):
        assert np.allclose(got[lane], total[2 * lane: 2 * lane + 2])
    # value index = token * 4 + head
    for lane in range(32):
        t, g0 = divmod(2 * lane, 4)
        assert t == lane >> 1 and g0 == 2 * (lane & 1)


def test_lane_dims_cover_the_row_once():
    dims = []
    for lane in range(32):
        half, chunk, part = lane >> 4, (lane >> 1) & 7, lane & 1
        byte = half * 128 + chunk * 16 + part * 8   # of the 256-byte 16-bit row
        dims.extend(range(byte // 2, byte // 2 + 4))
        assert dims[-4] == 4 * lane
    assert sorted(dims) == list(range(128))
