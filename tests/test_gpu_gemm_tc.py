"""The tensor-core projection GEMM (tcgen05, exact int8-limb activations) behind enx_matmul_q4 for
M >= 16 rows, at the model's projection shapes and config 1's M values, against the CPU oracle's
f64 linear (test/reference/quant.ts:95-112).

The kernel sums each 64-element block exactly in integers and rounds once per block, so apart
from a rare last-bit difference of the f64 sums the results equal the oracle's bit for bit; the
tests ask for BASELINE's tolerance everywhere and bit-identity on at least 99.9 % of outputs."""

import numpy as np
import pytest
import torch

from enargeia_b200 import kernels as K
from enargeia_b200.format import quantize_tensor

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-4, 1e-3


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run(x, t, bias, m, out_stride=None, out_offset=0):
    n, k = t.rows, t.cols
    stride = n if out_stride is None else out_stride
    out = torch.zeros(m * stride + out_offset, dtype=torch.float32, device="cuda")
    K.matmul_q4(dev(x), K.to_device_u32(t.packed), dev(t.scales), K.to_device_u32(t.zeros),
                None if bias is None else dev(bias), out, m, n, k, stride, out_offset)
    K.raw_check()  # synchronises; raises if a bounded device wait gave up
    return out.cpu().numpy()


def check(actual, expected):
    actual = np.asarray(actual, np.float64).reshape(-1)
    expected = np.asarray(expected, np.float64).reshape(-1)
    ratio = np.abs(actual - expected) / (ATOL + RTOL * np.abs(expected))
    i = int(np.argmax(ratio))
    assert ratio[i] <= 1.0, f"worst at {i}: {actual[i]} vs {expected[i]}"
    same = float(np.mean(actual == expected))
    assert same >= 0.999, f"only {same:.5f} bit-identical"


@pytest.mark.parametrize("m", [16, 64, 256])
@pytest.mark.parametrize("n,k", [(896, 896), (128, 896), (4864, 896), (896, 4864)])
def test_gemm_tc_projection_shapes(gpu, oracle, m, n, k):
    x = oracle.random_floats(m * k, 700 + m)
    t = quantize_tensor("w", oracle.random_floats(n * k, 701 + n).reshape(n, k), 4)
    b = oracle.random_floats(n, 702) if n in (896, 128) and k == 896 else None
    check(run(x, t, b, m), oracle.linear_q(t, x, b))


def test_gemm_tc_ragged_rows_and_tokens(gpu, oracle):
    m, n, k = 37, 200, 192  # neither a multiple of 32 tokens nor of 128 rows
    x = oracle.random_floats(m * k, 710)
    t = quantize_tensor("w", oracle.random_floats(n * k, 711).reshape(n, k), 4)
    check(run(x, t, oracle.random_floats(n, 712), m), oracle.linear_q(t, x, oracle.random_floats(n, 712)))


def test_gemm_tc_out_stride_and_offset(gpu, oracle):
    m, n, k = 32, 128, 128
    x = oracle.random_floats(m * k, 720)
    t = quantize_tensor("w", oracle.random_floats(n * k, 721).reshape(n, k), 4)
    out = run(x, t, None, m, out_stride=3 * n, out_offset=n)[: m * 3 * n].reshape(m, 3 * n)
    check(out[:, n:2 * n], oracle.linear_q(t, x))
    assert not out[:, :n].any() and not out[:, 2 * n:].any()


def test_gemm_tc_activation_extremes(gpu, oracle):
    """Blocks mixing magnitudes 2^-30 apart, zeros and exact powers of two (the limb split's
    fixed-point range edges)."""
    m, n, k = 16, 128, 256
    rng = np.random.default_rng(730)
    x = rng.standard_normal(m * k).astype(np.float32)
    x[::7] *= np.float32(2.0 ** -30)
    x[::11] = 0.0
    x[::13] = np.float32(2.0 ** 5)
    x[5 * k:6 * k] = 0.0  # an all-zero token
    t = quantize_tensor("w", oracle.random_floats(n * k, 731).reshape(n, k), 4)
    check(run(x, t, None, m), oracle.linear_q(t, x))


def test_gemm_tc_rows_match_decode_path(gpu, oracle):
    """A token's row of the M=16 tensor-core result equals the M=1 CUDA-core result (both round
    the exact block sums once)."""
    n, k = 896, 896
    x = oracle.random_floats(16 * k, 740)
    t = quantize_tensor("w", oracle.random_floats(n * k, 741).reshape(n, k), 4)
    many = run(x, t, None, 16).reshape(16, n)
    one = run(x[3 * k:4 * k], t, None, 1)
    assert float(np.mean(many[3] == one)) >= 0.999


def test_gemm_tc_is_deterministic(gpu, oracle):
    m, n, k = 64, 4864, 896
    x = oracle.random_floats(m * k, 750)
    t = quantize_tensor("w", oracle.random_floats(n * k, 751).reshape(n, k), 4)
    runs = [run(x, t, None, m) for _ in range(3)]
    for r in runs[1:]:
        np.testing.assert_array_equal(r, runs[0])
