"""Host-side check of the GPU sampler's top-p algorithm (enargeia_b200/csrc/k_sample.cu).

The kernel replaces the reference's 32 sequential bisection steps (src/kernels/sample.wgsl:
241-262) by four passes that each resolve 8 steps through a tree of midpoints.  This mirror of
that tree walk, in numpy, with the kernels' exact 62-bit fixed-point bucket masses, must land on exactly the threshold the oracle's sequential bisection
finds, for every distribution shape including ties."""

import numpy as np
import pytest

f32 = np.float32


def fx62(p):
    return np.rint(np.asarray(p, np.float64) * 2.0 ** 62).astype(np.uint64)


def tree_bisection(p: np.ndarray, top_p: float) -> float:
    lo, hi = f32(0.0), f32(1.0)
    for _ in range(4):
        L = np.zeros(256, f32)
        H = np.zeros(256, f32)
        mids = np.zeros(256, f32)
        thr = np.zeros(256, np.float64)
        L[1], H[1] = lo, hi
        for n in range(1, 256):
            mid = f32(f32(L[n] + H[n]) * f32(0.5))
            mids[n] = mid
            if n < 128:
                L[2 * n], H[2 * n] = L[n], mid
                L[2 * n + 1], H[2 * n + 1] = mid, H[n]
        rank = lambda n: (2 * (n - (1 << (n.bit_length() - 1))) + 1) << (7 - (n.bit_length() - 1))
        for n in range(1, 256):
            thr[rank(n)] = float(mids[n])
        b = np.searchsorted(thr[1:256], p, side="right")  # number of thresholds <= p
        M = np.zeros(256, np.uint64)  # 62-bit fixed-point masses, as the kernels sum them
        np.add.at(M, b, fx62(p))
        suffix = np.cumsum(M[::-1])[::-1]
        goal = fx62(float(f32(top_p)))
        n = 1
        l, h = lo, hi
        for _ in range(8):
            if suffix[rank(n)] < goal:
                h = mids[n]
                n = 2 * n
            else:
                l = mids[n]
                n = 2 * n + 1
        lo, hi = l, h
    return float(lo)


def _cases():
    rng = np.random.default_rng(11)
    yield "normal", rng.standard_normal(151936).astype(f32) * f32(0.6)
    yield "peaked", (rng.standard_normal(5000) * 8).astype(f32)
    t = np.zeros(4096, f32)
    t[:37] = 3.0  # a tied plateau at the top
    yield "ties", t
    yield "uniform", np.zeros(1000, f32)
    y = rng.standard_normal(20000).astype(f32)
    y[123] = 40.0  # one token holds almost all mass
    yield "spike", y


@pytest.mark.parametrize("top_p", [0.0, 0.1, 0.5, 0.9, 0.999])
@pytest.mark.parametrize("name,logits", list(_cases()))
def test_tree_equals_sequential_bisection(oracle, name, logits, top_p):
    T = f32(0.7)
    s = (logits / T).astype(f32)
    e = np.exp(s.astype(np.float64) - float(s.max()))
    p = e / e.sum()
    _, tr = oracle.sample(logits.copy(), [], float(T), top_p, 1.0, 0.5, trace=True)
    assert tree_bisection(p, top_p) == tr["threshold"]
