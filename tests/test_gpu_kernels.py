"""Raw libenx kernels on the GPU against the CPU oracle, at the reference's test shapes
(test/kernels/matmul_q4.test.ts, test/kernels/forward_ops.test.ts) and the model's shapes.

Tolerances: float kernels use the reference's FP32_TOLERANCE (1e-4 abs + 1e-4 rel,
test/reference/matmul.ts:462) against the f64-accumulating oracle; integer/byte work (f16
packing, sampled ids) is compared exactly."""

import numpy as np
import pytest
import torch

from enargeia_b200 import kernels as K
from enargeia_b200.format import quantize_tensor

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-4, 1e-4


def within(actual, expected, atol=ATOL, rtol=RTOL):
    actual = np.asarray(actual, np.float64).reshape(-1)
    expected = np.asarray(expected, np.float64).reshape(-1)
    err = np.abs(actual - expected)
    ratio = err / (atol + rtol * np.abs(expected))
    i = int(np.argmax(ratio)) if ratio.size else 0
    assert ratio.size == 0 or ratio[i] <= 1.0, f"worst at {i}: {actual[i]} vs {expected[i]} ({ratio[i]:.2f} of tol)"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def qdev(t):
    return K.to_device_u32(t.packed), dev(t.scales), K.to_device_u32(t.zeros)


def run_q4(x, t, bias, m, out_stride=None, out_offset=0, out_len=None):
    n, k = t.rows, t.cols
    stride = n if out_stride is None else out_stride
    out = torch.zeros(out_len if out_len else m * stride + out_offset, dtype=torch.float32, device="cuda")
    p, s, z = qdev(t)
    K.matmul_q4(dev(x), p, s, z, None if bias is None else dev(bias), out, m, n, k, stride, out_offset)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("n", [896, 128, 4864])
def test_matmul_q4_decode_shapes(gpu, oracle, n):
    k = 896
    x = oracle.random_floats(k, 41)
    t = quantize_tensor("w", oracle.random_floats(n * k, 42).reshape(n, k), 4)
    b = oracle.random_floats(n, 43)
    within(run_q4(x, t, b, 1), oracle.linear_q(t, x, b))


def test_matmul_q4_down_shape(gpu, oracle):
    n, k = 896, 4864
    x = oracle.random_floats(k, 44)
    t = quantize_tensor("w", oracle.random_floats(n * k, 45).reshape(n, k), 4)
    within(run_q4(x, t, None, 1), oracle.linear_q(t, x))


@pytest.mark.parametrize("m,n,k", [(15, 896, 896), (15, 128, 896), (4, 4864, 896), (64, 32, 64), (3, 5, 64),
                                   (8, 896, 4864), (2, 64, 128)])
def test_matmul_q4_prefill_shapes(gpu, oracle, m, n, k):
    x = oracle.random_floats(m * k, 11)
    t = quantize_tensor("w", oracle.random_floats(n * k, 12).reshape(n, k), 4)
    b = oracle.random_floats(n, 13)
    within(run_q4(x, t, b, m), oracle.linear_q(t, x, b))


def test_matmul_q4_out_offset_known_answer(gpu):
    k = 64
    t = quantize_tensor("w", np.full((2, k), 0.5, np.float32), 4)
    out = run_q4(np.ones(k, np.float32), t, None, 1, out_stride=6, out_offset=4, out_len=6)
    assert out[0] == 0 and abs(out[4] - 32) < 1e-3 and abs(out[5] - 32) < 1e-3


def test_matmul_decode_equals_prefill_row(gpu, oracle):
    n, k = 256, 192
    x = oracle.random_floats(k, 51)
    t = quantize_tensor("w", oracle.random_floats(n * k, 52).reshape(n, k), 4)
    one = run_q4(x, t, None, 1)
    many = run_q4(np.concatenate([x, x, x]), t, None, 3).reshape(3, n)
    np.testing.assert_array_equal(many[1], one)


def test_matmul_is_deterministic(gpu, oracle):
    n, k = 4864, 896
    x = oracle.random_floats(k, 61)
    t = quantize_tensor("w", oracle.random_floats(n * k, 62).reshape(n, k), 4)
    runs = [run_q4(x, t, None, 1) for _ in range(5)]
    for r in runs[1:]:
        np.testing.assert_array_equal(r, runs[0])


@pytest.mark.parametrize("rows", [151936, 1000, 37])
def test_lm_head_q8(gpu, oracle, rows):
    h = 896
    rng = np.random.default_rng(rows)
    w = (rng.standard_normal((rows, h), dtype=np.float32) * np.float32(0.02))
    t = quantize_tensor("e", w, 8)
    x = rng.standard_normal(h, dtype=np.float32)
    out = torch.zeros(rows, dtype=torch.float32, device="cuda")
    p, s, z = qdev(t)
    K.lm_head_q8(dev(x), p, s, z, out, rows, h)
    torch.cuda.synchronize()
    within(out.cpu().numpy(), oracle.linear_q(t, x))


@pytest.mark.parametrize("rows,seq,h", [(151936, 1, 896), (151936, 2, 896), (1000, 3, 896), (4099, 4, 896), (1000, 2, 128)])
def test_lm_head_q8_tensor_core_rows(gpu, oracle, rows, seq, h):
    """1-4 decode rows take the tensor-core head (exact activation limbs, int8 codes as stored):
    the reference's per-product double sum to within BASELINE's tolerance, bit-identical for all
    but rare last-bit roundings, and no bounded wait may have given up."""
    rng = np.random.default_rng(rows + seq)
    w = rng.standard_normal((rows, h), dtype=np.float32) * np.float32(0.02)
    t = quantize_tensor("e", w, 8)
    x = rng.standard_normal(seq * h, dtype=np.float32).reshape(seq, h)
    out = torch.zeros(seq * rows, dtype=torch.float32, device="cuda")
    p, s, z = qdev(t)
    xd = dev(x)
    d = K.EmbeddingDims(seq, h, 0, rows, 64, h // 64, rows, 0, min(rows, 65535), 0, 0, 0)
    K.call("enx_lm_head_q8", xd.data_ptr(), p.data_ptr(), s.data_ptr(), z.data_ptr(), out.data_ptr(), K.C.byref(d), None)
    K.raw_check()
    got = out.cpu().numpy().reshape(seq, rows)
    for i in range(seq):
        want = oracle.linear_q(t, x[i])
        within(got[i], want)
        assert np.mean(got[i] == want) >= 0.999


def test_embed_gather_q8(gpu, oracle):
    V, h = 5000, 896
    rng = np.random.default_rng(3)
    t = quantize_tensor("e", rng.standard_normal((V, h), dtype=np.float32) * np.float32(0.02), 8)
    ids = np.array([0, 4999, 17, 17, 2500], np.uint32)
    out = torch.zeros(len(ids) * h, dtype=torch.float32, device="cuda")
    p, s, z = qdev(t)
    K.embed_gather_q8(K.to_device_u32(ids), p, s, z, out, h, 0, V)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().reshape(len(ids), h), oracle.embed_q(t, ids))


def test_rmsnorm(gpu, oracle):
    x = np.random.default_rng(1).standard_normal(3 * 896).astype(np.float32)
    w = np.random.default_rng(2).standard_normal(896).astype(np.float32)
    out = torch.zeros_like(dev(x))
    K.rmsnorm(dev(x), dev(w), out, 3, 896)
    torch.cuda.synchronize()
    within(out.cpu().numpy(), oracle.rmsnorm(x.reshape(3, 896), w))


def test_rope_from_table(gpu, oracle):
    c, s = oracle.rope_table(64, 64, 1e6)
    x = oracle.random_floats(5 * 14 * 64, 8)
    out = torch.zeros_like(dev(x))
    K.rope(dev(x), out, dev(c), dev(s), 5, 14, 64, pos0=20)
    torch.cuda.synchronize()
    within(out.cpu().numpy(), oracle.rope(x, 14, 64, 1e6, pos_offset=20), atol=1e-6, rtol=1e-5)


def test_cache_pack_is_bit_exact(gpu, oracle):
    x = (np.random.default_rng(9).standard_normal(4096) * 3).astype(np.float32)
    dst = torch.zeros(4096 + 128, dtype=torch.int16, device="cuda")
    K.cache_pack(dev(x), dst, 4096, 128)
    torch.cuda.synchronize()
    got = dst.cpu().numpy().view(np.uint16)[128:]
    np.testing.assert_array_equal(got, oracle.f32_to_f16_bits(x))


def test_silu_mul_and_add(gpu, oracle):
    g = np.random.default_rng(4).standard_normal(4864).astype(np.float32) * 4
    u = np.random.default_rng(5).standard_normal(4864).astype(np.float32)
    out = torch.zeros_like(dev(g))
    K.silu_mul(dev(g), dev(u), out)
    torch.cuda.synchronize()
    within(out.cpu().numpy(), oracle.silu_mul(g, u), atol=1e-6, rtol=1e-6)
    K.add(dev(g), dev(u), out)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), g + u)


@pytest.mark.parametrize("position", [0, 1, 63, 64, 95, 700, 2047])
def test_attn_decode(gpu, oracle, position):
    heads, kvh, hd = 14, 2, 64
    n = position + 1
    rng = np.random.default_rng(position)
    q = rng.standard_normal(heads * hd).astype(np.float32)
    kb = oracle.f32_to_f16_bits(rng.standard_normal(n * kvh * hd).astype(np.float32))
    vb = oracle.f32_to_f16_bits(rng.standard_normal(n * kvh * hd).astype(np.float32))
    out = torch.zeros(heads * hd, dtype=torch.float32, device="cuda")
    K.attn_decode(dev(q), dev(kb.view(np.int16)), dev(vb.view(np.int16)), out, position, heads, kvh, hd)
    torch.cuda.synchronize()
    within(out.cpu().numpy(), oracle.attention_f16(q, kb, vb, position, heads, kvh, hd), atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("queries,begin,hd", [(16, 0, 64), (37, 100, 64), (5, 3, 32)])
def test_attn_prefill(gpu, oracle, queries, begin, hd):
    heads, kvh = (14, 2) if hd == 64 else (4, 2)
    n = begin + queries
    rng = np.random.default_rng(queries)
    q = rng.standard_normal(queries * heads * hd).astype(np.float32)
    kb = oracle.f32_to_f16_bits(rng.standard_normal(n * kvh * hd).astype(np.float32))
    vb = oracle.f32_to_f16_bits(rng.standard_normal(n * kvh * hd).astype(np.float32))
    out = torch.zeros(queries * heads * hd, dtype=torch.float32, device="cuda")
    K.attn_prefill(dev(q), dev(kb.view(np.int16)), dev(vb.view(np.int16)), out, queries, begin, heads, kvh, hd)
    torch.cuda.synchronize()
    within(out.cpu().numpy(), oracle.attention_f16(q, kb, vb, begin, heads, kvh, hd), atol=1e-5, rtol=1e-4)


def _sample_gpu(logits, hist, t, p, rp, r):
    lg = dev(logits.copy())
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    h = K.to_device_u32(np.asarray(hist, np.uint32)) if len(hist) else None
    K.sample(lg, h, out, t, p, rp, r)
    torch.cuda.synchronize()
    return int(out.item()), lg.cpu().numpy()


@pytest.mark.parametrize("V", [151936, 1000, 7])
def test_sampler_matches_oracle(gpu, oracle, V):
    rng = np.random.default_rng(V)
    mism = 0
    for trial in range(40):
        logits = (rng.standard_normal(V) * rng.choice([0.3, 0.6, 2.0, 8.0])).astype(np.float32)
        hist = rng.integers(0, V + 5, size=rng.integers(0, 2048)).astype(np.uint32)
        t, p, rp = [(0.7, 0.9, 1.1), (1.0, 1.0, 1.0), (0.0, 1.0, 1.3), (0.5, 0.5, 1.0), (1.3, 0.99, 1.05)][trial % 5]
        r = float(np.float32(rng.random()))
        ref = logits.copy()
        want, tr = oracle.sample(ref, hist, t, p, rp, r, trace=True)
        got, lg = _sample_gpu(logits, hist, t, p, rp, r)
        np.testing.assert_array_equal(lg, ref)  # the in-place penalty is bit-exact
        if got != want:
            mism += 1
            # a mismatch is only acceptable when a decision margin is at double rounding level
            assert min(tr["cross_margin"], tr["prev_margin"], tr["min_mass_margin"]) < 1e-12, (trial, got, want, tr)
    assert mism == 0


def test_sampler_greedy_ties_lowest_index(gpu):
    logits = np.zeros(151936, np.float32)
    logits[[500, 7, 90000]] = 3.0
    got, _ = _sample_gpu(logits, [], 0.0, 1.0, 1.0, 0.5)
    assert got == 7


def test_sampler_batched_rows(gpu, oracle):
    V, B = 151936, 4
    rng = np.random.default_rng(77)
    logits = (rng.standard_normal((B, V)) * 0.6).astype(np.float32)
    hist = rng.integers(0, V, size=(B, 64)).astype(np.uint32)
    lens = np.array([64, 10, 0, 33], np.uint32)
    params = [(0.7, 0.9, 1.1, 0.25), (0.0, 1.0, 1.1, 0.5), (1.0, 0.5, 1.0, 0.75), (0.7, 0.9, 1.1, 0.999)]
    out = torch.zeros(B, dtype=torch.int32, device="cuda")
    lg = dev(logits.copy())
    K.sample_batched(lg, K.to_device_u32(hist), K.to_device_u32(lens), K.sampling_rows(params), out)
    torch.cuda.synchronize()
    for b in range(B):
        ref = logits[b].copy()
        want = oracle.sample(ref, hist[b, : lens[b]], *params[b][:3], float(np.float32(params[b][3])))
        assert int(out[b].item()) == want
