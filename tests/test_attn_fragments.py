"""Host emulation of the f64 tensor-core fragment mapping the many-token attention kernels use
(enargeia_b200/csrc/k_decode.cu: k_attn_scores_split, k_attn_apply_split), checked against plain
matrix products.  mma.sync m8n8k4 .f64 computes D[8x8] += A[8x4] B[4x8] with, per lane:
A[lane / 4][lane % 4], B[lane % 4][lane / 4], D[lane / 4][2 (lane % 4) + {0, 1}].

* scores: A = query rows (heads), B = K rows (positions); lane k-slot q owns dimensions
  q hd/4 .. q hd/4 + hd/4 - 1, and step s uses dimension q hd/4 + s in both operands;
* weighted V: A = weights (head x 4 positions), B = V (4 positions x 8 dims); D column c of tile
  n holds dimension c hd/8 + n, so a lane (B column lane / 4) reads hd/8 contiguous values."""

import numpy as np
import pytest


def mma(D, A_lane, B_lane):
    """One m8n8k4 step from per-lane operand values: D[8][8] += A B."""
    A = np.zeros((8, 4))
    B = np.zeros((4, 8))
    for lane in range(32):
        A[lane // 4, lane % 4] = A_lane[lane]
        B[lane % 4, lane // 4] = B_lane[lane]
    D += A @ B


@pytest.mark.parametrize("hd", [32, 64])
@pytest.mark.parametrize("group", [2, 7])
def test_scores_fragments(hd, group):
    rng = np.random.default_rng(hd + group)
    q = np.zeros((8, hd))
    q[:group] = rng.standard_normal((group, hd))  # rows past the group are zero
    k = rng.standard_normal((8, hd))  # 8 positions
    steps = hd // 4
    D = np.zeros((8, 8))
    for s in range(steps):
        a = [q[lane // 4, (lane % 4) * steps + s] for lane in range(32)]  # A: head row, k-slot dim
        b = [k[lane // 4, (lane % 4) * steps + s] for lane in range(32)]  # B: position column
        mma(D, a, b)
    np.testing.assert_allclose(D[:group], (q @ k.T)[:group], rtol=1e-12, atol=1e-12)
    # D columns 2 (lane % 4) + e are positions p0 + 2 quad + e: the kernel's store mapping
    for lane in range(32):
        row, quad = lane // 4, lane % 4
        for e in range(2):
            assert D[row, 2 * quad + e] == pytest.approx((q @ k.T)[row, 2 * quad + e], abs=1e-12)


@pytest.mark.parametrize("hd", [32, 64])
@pytest.mark.parametrize("group", [2, 7])
def test_weighted_v_fragments(hd, group):
    rng = np.random.default_rng(100 + hd + group)
    npos = 16
    w = np.zeros((8, npos))
    w[:group] = rng.random((group, npos))
    v = rng.standard_normal((npos, hd))
    tiles = hd // 8
    D = [np.zeros((8, 8)) for _ in range(tiles)]
    for k0 in range(0, npos, 4):
        a = [w[lane // 4, k0 + lane % 4] for lane in range(32)]  # A: head, position k0 + quad
        for n in range(tiles):
            # B column c = lane / 4 is dimension c * tiles + n of position k0 + lane % 4
            b = [v[k0 + lane % 4, (lane // 4) * tiles + n] for lane in range(32)]
            mma(D[n], a, b)
    out = np.zeros((8, hd))
    for n in range(tiles):
        for c in range(8):
            out[:, c * tiles + n] = D[n][:, c]  # the kernel's red[warp][row][c * tiles + n]
    np.testing.assert_allclose(out[:group], (w @ v)[:group], rtol=1e-12, atol=1e-12)
    # a lane's B values over the tiles are hd/8 contiguous dimensions of one position
    for lane in range(32):
        dims = [(lane // 4) * tiles + n for n in range(tiles)]
        assert dims == list(range(dims[0], dims[0] + tiles))
