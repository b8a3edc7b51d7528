"""Batched decode (config 4's shape at test scale): more than four independent sequences per
enx_decode_step / enx_decode_loop, each at its own position with its own prompt, sampling
parameters and seed, against one CPU oracle session per sequence.  From 16 sequences the
projections and the tied head run on the tensor-core GEMM; 5-15 use the CUDA-core GEMM.

Ids must be identical per sequence; logits within BASELINE's 1e-3 rel / 1e-4 abs and bit-identical
on at least 99.9 % (the device sums every block exactly or in double and rounds where the
reference rounds)."""

import numpy as np
import pytest

from conftest import GOLDEN
from enargeia_b200.checkpoint import TINY
from enargeia_b200.session import APP_SAMPLING, GREEDY, Model, SamplingParams, mulberry32

pytestmark = pytest.mark.gpu


def within(actual, expected, atol=1e-4, rtol=1e-3, min_identical=0.999):
    err = np.abs(actual.astype(np.float64) - expected)
    ratio = err / (atol + rtol * np.abs(expected))
    i = int(np.argmax(ratio))
    assert ratio[i] <= 1.0, f"worst logit {i}: {actual[i]} vs {expected[i]}"
    assert float(np.mean(actual == expected)) >= min_identical


def params_for(b):
    return [GREEDY, APP_SAMPLING, SamplingParams(1.0, 1.0, 1.0), SamplingParams(0.5, 0.8, 1.3)][b % 4]


def setup(oracle, tiny_file, B, ctx):
    m = Model(TINY).load(GOLDEN / "tiny_q8.enargeia").kv_alloc(ctx, B)
    rng = np.random.default_rng(900 + B)
    seqs = []
    for b in range(B):
        prompt = [int(v) for v in rng.integers(0, TINY.vocab, int(rng.integers(5, 30)))]
        p = params_for(b)
        om = oracle.OracleModel(tiny_file, TINY, ctx)
        os_ = oracle.OracleSession(om, p.temperature, p.top_p, p.repetition_penalty, seed=1000 + b)
        draw = mulberry32(1000 + b)
        m.prefill(b, prompt)
        ol = om.prefill(prompt)
        within(m.logits(b), ol)
        os_.tokens = list(prompt)
        want = os_._sample(ol.copy())
        got = m.sample_prefill(b, p, float(np.float32(draw())))
        assert got == want, (b, got, want)
        os_.tokens.append(want)
        seqs.append((p, om, os_, draw, want))
    return m, seqs


@pytest.mark.parametrize("B", [6, 20])
def test_batched_decode_matches_per_sequence_oracle(gpu, oracle, tiny_file, B):
    m, seqs = setup(oracle, tiny_file, B, 64)
    toks = [s[4] for s in seqs]
    params = [s[0] for s in seqs]
    for step in range(12):
        randoms = [float(np.float32(s[3]())) for s in seqs]
        got = m.decode_step(toks, params, randoms)
        for b, (p, om, os_, draw, _) in enumerate(seqs):
            ol = om.decode(toks[b])
            olp = ol.copy()
            want = os_._sample(olp)
            within(m.logits(b), olp)
            assert got[b] == want, (step, b, got[b], want)
            os_.tokens.append(want)
        toks = got
    m.close()


def test_batched_loop_equals_batched_steps(gpu, oracle, tiny_file):
    """The device-fed loop (sampled id feeds the next step on the GPU) gives the same ids as the
    per-step API over 32 sequences."""
    B, steps = 32, 10
    runs = []
    for use_loop in (False, True):
        m, seqs = setup(oracle, tiny_file, B, 64)
        params = [s[0] for s in seqs]
        first = [s[4] for s in seqs]
        randoms = np.array([[np.float32(s[3]()) for s in seqs] for _ in range(steps)], np.float32)
        if use_loop:
            ids = m.decode_loop(first, params, randoms, steps)
        else:
            toks, ids = first, []
            for i in range(steps):
                toks = m.decode_step(toks, params, list(randoms[i]))
                ids.append(toks)
            ids = np.array(ids)
        runs.append(np.asarray(ids))
        m.close()
    np.testing.assert_array_equal(runs[0], runs[1])


def test_batched_first_four_equal_small_batches(gpu, oracle, tiny_file):
    """Sequences decoded in a batch of 24 get the ids they get in batches of one."""
    B, steps = 24, 6
    m, seqs = setup(oracle, tiny_file, B, 64)
    toks = [s[4] for s in seqs]
    params = [s[0] for s in seqs]
    rand = [[float(np.float32(s[3]())) for s in seqs] for _ in range(steps)]
    batched = []
    for i in range(steps):
        toks = m.decode_step(toks, params, rand[i])
        batched.append(toks)
    m.close()
    for b in range(3):
        p, om, os_, draw, first = seqs[b]
        m1 = Model(TINY).load(GOLDEN / "tiny_q8.enargeia").kv_alloc(64, 1)
        rng = np.random.default_rng(900 + B)
        prompts = []
        for bb in range(B):
            prompts.append([int(v) for v in rng.integers(0, TINY.vocab, int(rng.integers(5, 30)))])
        m1.prefill(0, prompts[b])
        tok = first
        for i in range(steps):
            tok = m1.decode_step([tok], [p], [rand[i][b]])[0]
            assert tok == batched[i][b], (b, i)
        m1.close()
