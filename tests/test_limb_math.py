"""Host restatement of the integer arithmetic the tensor-core projection GEMM relies on
(enargeia_b200/csrc/k_gemm_tc.cu), checked exactly in Python integers:

* k_limbs: the per-row exponent F = 46 - e (|x| < 2^e for the row's largest |x|), X = rint(x 2^F)
  with |X| < 2^46, and six balanced base-256 digits that rebuild X;
* the MMA + epilogue join: per 64-element block the int32 limb sums D_l = sum_k a_k d_lk, the
  pairs D_2i + 256 D_2i+1 fitting 32 bits, and the 64-bit join equal to sum_k a_k X_k, for int4
  (a = q - z, |a| <= 15) and int8 (a = q, 0..255) codes at their extremes;
* k_codes_i8: the per-byte q - z through ((q | 0x80) - z) ^ 0x80 for every int4 code and zero;
* the slot order: int4 slot j < 32 holds element 8(j / 4) + 2(j % 4), slot 32 + j the next one.

These are the facts the GPU parity tests (tests/test_gpu_gemm_tc.py) exercise end to end."""

import numpy as np
import pytest


def row_exponent(x: np.ndarray) -> int:
    amax = float(np.max(np.abs(x))) if x.size else 0.0
    if amax == 0.0:
        return 46
    bits = np.array([amax], np.float32).view(np.uint32)[0]
    e = int((bits >> 23) & 0xFF) - 126
    return 46 - e


def to_x(x: np.ndarray, F: int) -> list:
    return [int(np.rint(np.float64(v) * 2.0 ** F)) for v in x]


def limbs(X: int) -> list:
    u = (X + 0x808080808080) & ((1 << 64) - 1)
    return [((u >> (8 * l)) & 0xFF) - 128 for l in range(6)]


def slot_element(bits: int, j: int) -> int:
    if bits == 8:
        return j
    return 8 * (j // 4) + 2 * (j % 4) if j < 32 else 8 * ((j - 32) // 4) + 2 * ((j - 32) % 4) + 1


def rows():
    rng = np.random.default_rng(17)
    yield rng.standard_normal(896).astype(np.float32)
    y = rng.standard_normal(896).astype(np.float32)
    y[::7] *= np.float32(2.0 ** -30)  # tiny elements next to normal ones
    y[3] = np.float32(2.0 ** 5)  # an exact power of two as the row maximum
    yield y
    yield np.zeros(128, np.float32)
    yield np.full(64, np.float32(-3.0e38))  # the largest magnitudes a float holds
    yield np.full(64, np.float32(1.0e-40))  # subnormal floats only


@pytest.mark.parametrize("x", list(rows()))
def test_limbs_rebuild_the_scaled_row(x):
    F = row_exponent(x)
    Xs = to_x(x, F)
    amax = float(np.max(np.abs(x)))
    for v, X in zip(x, Xs):
        assert abs(X) < 2 ** 46
        d = limbs(X)
        assert all(-128 <= di <= 127 for di in d)
        assert sum(di * 256 ** l for l, di in enumerate(d)) == X
        if v != 0 and abs(float(v)) >= amax * 2.0 ** -22:
            assert X * 2.0 ** -F == float(v)  # exact: no bits of x lost


@pytest.mark.parametrize("bits", [4, 8])
def test_block_join_is_exact_and_in_range(bits):
    rng = np.random.default_rng(23 + bits)
    amax_code = 15 if bits == 4 else 255
    # codes at their extremes and at random, X at the top of the 46-bit range and at random
    for case in range(6):
        if case == 0:
            a = [amax_code] * 64
            X = [2 ** 46 - 1] * 64
        elif case == 1:
            a = [-amax_code if bits == 4 else 0] * 64
            X = [-(2 ** 46 - 1)] * 64
        else:
            a = [int(v) for v in rng.integers(-amax_code if bits == 4 else 0, amax_code + 1, 64)]
            X = [int(v) for v in rng.integers(-(2 ** 46) + 1, 2 ** 46, 64)]
        d = [limbs(v) for v in X]
        D = [sum(a[k] * d[k][l] for k in range(64)) for l in range(6)]  # the int32 MMA sums
        assert all(-(2 ** 31) <= v < 2 ** 31 for v in D)
        pairs = [D[0] + 256 * D[1], D[2] + 256 * D[3], D[4] + 256 * D[5]]
        assert all(-(2 ** 31) <= v < 2 ** 31 for v in pairs)  # each pair fits 32 bits
        T = pairs[0] + pairs[1] * 65536 + pairs[2] * 2 ** 32
        assert T == sum(a[k] * X[k] for k in range(64))
        assert -(2 ** 63) <= T < 2 ** 63


def test_signed_code_bytes_for_every_int4_code_and_zero():
    for q in range(16):
        for z in range(16):
            word = q * 0x01010101
            zz = z * 0x01010101
            r = (((word & 0x0F0F0F0F) | 0x80808080) - zz) & 0xFFFFFFFF
            r ^= 0x80808080
            for byte in range(4):
                b = (r >> (8 * byte)) & 0xFF
                assert (b - 256 if b >= 128 else b) == q - z


def test_slot_order_matches_the_nibble_unpack():
    # a block's 32 packed bytes: byte w*4 + i holds elements 8w + 2i (low nibble) and 8w + 2i + 1
    slots = [slot_element(4, j) for j in range(64)]
    assert sorted(slots) == list(range(64))
    for w in range(8):
        for i in range(4):
            assert slots[4 * w + i] == 8 * w + 2 * i  # low nibbles: k-bytes 0..31
            assert slots[32 + 4 * w + i] == 8 * w + 2 * i + 1  # high nibbles: k-bytes 32..63
    assert [slot_element(8, j) for j in range(64)] == list(range(64))
