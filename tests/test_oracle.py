"""The CPU oracle against the reference's own known answers and properties.

Cases follow test/kernels/forward_ops.test.ts, test/kernels/matmul_q4.test.ts and
test/parity/session.test.ts; the model-level properties run on the TINY random-init model."""

import numpy as np
import pytest

from enargeia_b200.checkpoint import TINY
from enargeia_b200.format import quantize_tensor


def test_mulberry32_matches_python_session_rng(oracle):
    from enargeia_b200.session import mulberry32

    for seed in (0, 1, 0x5EED, 0xFFFFFFFF, 123456789):
        r = mulberry32(seed)
        np.testing.assert_array_equal(oracle.mulberry32(seed, 50), [r() for _ in range(50)])


def test_random_floats_range(oracle):
    v = oracle.random_floats(10000, 3)
    assert v.min() >= -0.5 and v.max() < 0.5


def test_linear_q4_equals_f32_over_dequantised(oracle):
    x = oracle.random_floats(8 * 128, 21).reshape(8, 128)
    q = quantize_tensor("w", oracle.random_floats(64 * 128, 22).reshape(64, 128), 4)
    got = oracle.linear_q(q, x).reshape(8, 64)
    want = x.astype(np.float64) @ q.dequantize().astype(np.float64).T
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)


def test_out_offset_known_answer(oracle):
    # matmul_q4.test.ts:181-195: ones . 0.5-constant rows of 64 = 32, written at outOffset 4
    k = 64
    q = quantize_tensor("w", np.full((2, k), 0.5, np.float32), 4)
    out = np.zeros(6, np.float32)
    oracle.linear_q(q, np.ones(k, np.float32), out_stride=6, out_offset=4, out=out)
    assert out[0] == 0 and abs(out[4] - 32) < 1e-3 and abs(out[5] - 32) < 1e-3


def test_rmsnorm_uses_mean_not_sum(oracle):
    x = np.full(896, 2.0, np.float32)
    y = oracle.rmsnorm(x, np.ones(896, np.float32))
    np.testing.assert_allclose(y, 1.0, rtol=1e-5)


def test_rope_position_zero_is_identity(oracle):
    x = oracle.random_floats(2 * 64, 9)
    np.testing.assert_array_equal(oracle.rope(x, 2, 64, pos_offset=0), x)


def test_rope_rotates_halves_not_neighbours(oracle):
    x = np.zeros(64, np.float32)
    x[0] = 1.0  # pairs with element 32
    y = oracle.rope(x, 1, 64, theta=1e6, pos_offset=1)
    assert abs(y[0] - np.cos(1.0)) < 1e-6 and abs(y[32] - np.sin(1.0)) < 1e-6
    assert y[1] == 0.0


def test_rope_table_matches_direct(oracle):
    c, s = oracle.rope_table(40, 64, 1e6)
    x = oracle.random_floats(64, 4)
    y = oracle.rope(x, 1, 64, 1e6, pos_offset=37)
    a, b = x[:32].astype(np.float64), x[32:].astype(np.float64)
    np.testing.assert_allclose(y[:32], a * c[37] - b * s[37], atol=1e-6)


def test_argmax_lowest_index_wins_ties(oracle):
    x = np.array([1, 5, 3, 5, 5], np.float32)
    assert oracle.argmax(x) == 1


def test_f16_rounding_is_round_to_nearest_even(oracle):
    import numpy as np
    v = np.array([1.0, 1 + 2**-11, 1 + 3 * 2**-11, 65504, 65520, 1e-8, -2.5e-5, 6.1e-5, np.inf, -0.0],
                 np.float32)
    with np.errstate(over="ignore"):
        np.testing.assert_array_equal(oracle.f32_to_f16_bits(v), v.astype(np.float16).view(np.uint16))
    r = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * np.float32(3)
    np.testing.assert_array_equal(oracle.f32_to_f16_bits(r), r.astype(np.float16).view(np.uint16))


def _attn_full(q, k, v, heads, kv_heads, hd):
    """Dense causal attention in f64 from the f16-rounded caches, no cache tricks."""
    S = q.shape[0]
    g = heads // kv_heads
    out = np.zeros((S, heads * hd))
    for h in range(heads):
        kv = h // g
        qh = q[:, h * hd:(h + 1) * hd].astype(np.float64)
        kh = k[:, kv * hd:(kv + 1) * hd].astype(np.float64)
        vh = v[:, kv * hd:(kv + 1) * hd].astype(np.float64)
        sc = qh @ kh.T / np.sqrt(hd)
        sc[np.triu_indices(S, 1)] = -np.inf
        w = np.exp(sc - sc.max(1, keepdims=True))
        w /= w.sum(1, keepdims=True)
        out[:, h * hd:(h + 1) * hd] = w @ vh
    return out


def test_attention_gqa_contiguous_grouping(oracle):
    heads, kvh, hd, S = 14, 2, 64, 9
    q = oracle.random_floats(S * heads * hd, 1).reshape(S, heads * hd)
    k = oracle.random_floats(S * kvh * hd, 2).reshape(S, kvh * hd)
    v = oracle.random_floats(S * kvh * hd, 3).reshape(S, kvh * hd)
    kb, vb = oracle.f32_to_f16_bits(k), oracle.f32_to_f16_bits(v)
    got = oracle.attention_f16(q, kb, vb, 0, heads, kvh, hd)
    want = _attn_full(q, kb.view(np.float16).astype(np.float32), vb.view(np.float16).astype(np.float32), heads, kvh, hd)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)


def test_attention_chunked_equals_full(oracle):
    heads, kvh, hd, S = 4, 2, 32, 12
    q = oracle.random_floats(S * heads * hd, 4).reshape(S, heads * hd)
    kb = oracle.f32_to_f16_bits(oracle.random_floats(S * kvh * hd, 5))
    vb = oracle.f32_to_f16_bits(oracle.random_floats(S * kvh * hd, 6))
    full = oracle.attention_f16(q, kb, vb, 0, heads, kvh, hd)
    part = oracle.attention_f16(q[7:], kb, vb, 7, heads, kvh, hd)
    np.testing.assert_array_equal(full[7:], part)


# --- model-level properties (test/parity/session.test.ts), on the TINY random-init model

def _model(oracle, f, ctx=128):
    return oracle.OracleModel(f, TINY, ctx)


def test_cached_decode_equals_recompute(oracle, tiny_file):
    ids = np.random.default_rng(1).integers(0, TINY.vocab, 24)
    m1 = _model(oracle, tiny_file)
    full = m1.prefill(ids)
    m2 = _model(oracle, tiny_file)
    m2.prefill(ids[:10])
    for t in ids[10:-1]:
        m2.decode(t)
    step = m2.decode(ids[-1])
    np.testing.assert_array_equal(full, step)


@pytest.mark.parametrize("chunk", [64, 16, 7])
def test_chunk_size_invariance(oracle, tiny_file, chunk):
    ids = np.random.default_rng(2).integers(0, TINY.vocab, 40)
    a = _model(oracle, tiny_file).prefill(ids, chunk=256)
    b = _model(oracle, tiny_file).prefill(ids, chunk=chunk)
    np.testing.assert_array_equal(a, b)


def test_context_exhausted_raises(oracle, tiny_file):
    m = _model(oracle, tiny_file, ctx=8)
    m.prefill(np.arange(8))
    with pytest.raises(oracle.RangeError):
        m.decode(1)


def _gen(oracle, f, prompt, n, t, p, rp, seed):
    s = oracle.OracleSession(_model(oracle, f), t, p, rp, seed)
    return s.generate(list(prompt), n)


def test_same_seed_same_ids(oracle, tiny_file):
    pr = np.random.default_rng(3).integers(0, TINY.vocab, 16)
    a = _gen(oracle, tiny_file, pr, 20, 0.7, 0.9, 1.1, 7)
    b = _gen(oracle, tiny_file, pr, 20, 0.7, 0.9, 1.1, 7)
    c = _gen(oracle, tiny_file, pr, 20, 0.7, 0.9, 1.1, 8)
    assert a == b and a != c


def test_low_temperature_full_nucleus_equals_greedy(oracle, tiny_file):
    pr = np.random.default_rng(4).integers(0, TINY.vocab, 16)
    g = _gen(oracle, tiny_file, pr, 12, 0.0, 1.0, 1.0, 1)
    s = _gen(oracle, tiny_file, pr, 12, 0.01, 1.0, 1.0, 1)
    assert g == s


def test_penalty_changes_output(oracle, tiny_file):
    pr = np.random.default_rng(5).integers(0, TINY.vocab, 16)
    # session.test.ts uses 1.5 on the real model; random-init logits put one token far ahead,
    # so the same property needs a stronger penalty here
    a = _gen(oracle, tiny_file, pr, 24, 0.0, 1.0, 1.0, 1)
    b = _gen(oracle, tiny_file, pr, 24, 0.0, 1.0, 3.0, 1)
    assert a != b


def test_penalty_first_occurrence_only(oracle):
    logits = np.array([2.0, -2.0, 1.0, 0.5], np.float32)
    oracle.sample(logits, [0, 1, 0, 0, 1, 9], 0.0, 1.0, 2.0, 0.3)  # 9 is out of vocab: ignored
    np.testing.assert_array_equal(logits, [1.0, -4.0, 1.0, 0.5])


def test_sampler_fallback_and_draw_order(oracle):
    # uniform distribution, top_p 1: the draw at random r picks id floor(r * V)
    V = 1000
    for r in (0.0, 0.1234, 0.5, 0.9999):
        logits = np.zeros(V, np.float32)
        tok = oracle.sample(logits, [], 1.0, 1.0, 1.0, r)
        assert tok == min(int(np.ceil(r * V)) - 1 if r > 0 else 0, V - 1) or tok == int(r * V)


def test_nll_matches_the_harness_formula(oracle):
    """-log softmax[target] of test/parity/quality.test.ts:93-99 (max of the floats, double sum)."""
    rng = np.random.default_rng(31)
    for scale in (0.5, 3.0, 30.0):
        lg = (rng.standard_normal(5000) * scale).astype(np.float32)
        t = int(rng.integers(0, lg.size))
        m = float(lg.max())
        s = 0.0
        for v in lg.astype(np.float64):
            s += np.exp(v - m)
        want = -((float(lg[t]) - m) - np.log(s))
        assert abs(oracle.nll(lg, t) - want) <= 1e-12 * abs(want) + 1e-12
