"""Parity at the context lengths of BASELINE configs 3 and 4, against the CPU oracle.

- the many-token attention (`enx_attn_prefill`) with 256 queries against up to 2048 keys, so the
  128-position score splits, the 512-position weighted-V splits and their in-order combine all
  run (ref src/kernels/cache_variants.ts:81-144, causal mask `j > i + queryBegin`);
- a 600-id prompt through the full-size config-0 model in 256-query chunks (three chunks: the
  causal mask of src/model/graph.ts:436-459 across chunk boundaries), every layer's f16 cache,
  the last-row logits and a few decode steps;
- batched decode of 16 sequences (tensor-core projections and head) of the mid-size model from
  prompts of 520-1000 ids decoded past position 1024, with per-sequence sampling and seeds.

Tolerances are BASELINE's: logits within 1e-3 rel / 1e-4 abs with at least 99.9 % bit-identical,
ids identical, cached f16 values identical except rare last-bit ties (at most one f16 ulp)."""

import os
from pathlib import Path

import numpy as np
import pytest
import torch

from enargeia_b200 import kernels as K
from enargeia_b200.checkpoint import QWEN2_0_5B, SMALL, build_model_file
from enargeia_b200.format import read_enargeia
from enargeia_b200.session import APP_SAMPLING, GREEDY, Model, SamplingParams, mulberry32

pytestmark = pytest.mark.gpu

SEED = 20251201  # the bench model
MODEL = Path(os.environ.get("ENX_MODEL_DIR", "/tmp/enx_models")) / f"qwen2.5-0.5b-random-s{SEED}-q4q8.enargeia"


def within(actual, expected, atol=1e-4, rtol=1e-3, min_identical=0.999):
    actual = np.asarray(actual, np.float32).reshape(-1)
    expected = np.asarray(expected, np.float32).reshape(-1)
    err = np.abs(actual.astype(np.float64) - expected)
    ratio = err / (atol + rtol * np.abs(expected.astype(np.float64)))
    i = int(np.argmax(ratio))
    assert ratio[i] <= 1.0, f"worst {i}: {actual[i]} vs {expected[i]} ({ratio[i]:.2f} of tol)"
    same = float(np.mean(actual == expected))
    assert same >= min_identical, f"only {same:.5f} bit-identical"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("begin", [0, 768, 1792])
def test_attn_prefill_chunk_against_2048_keys(gpu, oracle, begin):
    """One 256-query chunk at queryBegin = begin over begin + 256 cached keys."""
    heads, kvh, hd, queries = 14, 2, 64, 256
    n = begin + queries
    rng = np.random.default_rng(7000 + begin)
    q = rng.standard_normal(queries * heads * hd).astype(np.float32)
    kb = oracle.f32_to_f16_bits(rng.standard_normal(n * kvh * hd).astype(np.float32))
    vb = oracle.f32_to_f16_bits(rng.standard_normal(n * kvh * hd).astype(np.float32))
    out = torch.zeros(queries * heads * hd, dtype=torch.float32, device="cuda")
    K.attn_prefill(dev(q), dev(kb.view(np.int16)), dev(vb.view(np.int16)), out, queries, begin, heads, kvh, hd)
    torch.cuda.synchronize()
    want = oracle.attention_f16(q, kb, vb, begin, heads, kvh, hd)
    within(out.cpu().numpy(), want, atol=1e-5, rtol=1e-4)


def _copy_device(ptr: int, host: np.ndarray) -> None:
    from cuda.bindings import runtime as rt

    (err,) = rt.cudaMemcpy(host.ctypes.data, ptr, host.nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert int(err) == 0, err


def _check_cache(m, om, layers, n, kv_dim, seq=0):
    for layer in range(layers):
        kp, vp = m.kv_view(seq, layer)
        ok, ov = om.kv(layer)
        for ptr, ref in ((kp, ok), (vp, ov)):
            got = np.empty(n * kv_dim, np.uint16)
            _copy_device(ptr, got)
            diff = got != ref[: n * kv_dim]
            assert diff.mean() < 1e-3, (layer, int(diff.sum()))
            if diff.any():
                a = got[diff].view(np.float16).astype(np.float32)
                b = ref[: n * kv_dim][diff].view(np.float16).astype(np.float32)
                assert np.all(np.abs(a - b) <= np.abs(b) * 2.0**-10 + 1e-7), layer


def test_full_model_prefill_600_in_256_chunks(gpu, oracle):
    path = build_model_file(QWEN2_0_5B, SEED, MODEL)
    f = read_enargeia(path)
    cfg = QWEN2_0_5B
    n, ctx = 600, 608
    prompt = [int(v) for v in np.random.default_rng(3000).integers(0, cfg.vocab, n)]
    m = Model(cfg).load(path).kv_alloc(ctx)
    om = oracle.OracleModel(f, cfg, ctx)
    m.prefill(0, prompt, 256)
    want = om.prefill(prompt, 256)
    within(m.logits(), want)
    _check_cache(m, om, cfg.layers, n, cfg.kv_dim)
    tok = int(np.argmax(want))
    for step in range(4):  # decode continues from the chunked cache
        got = m.decode_step([tok], [GREEDY], [0.5])[0]
        ol = om.decode(tok)
        within(m.logits(), ol)
        want_id = oracle.argmax(ol)
        assert got == want_id, (step, got, want_id)
        tok = got
    m.close()


def test_batched_decode_16_past_1024(gpu, oracle, tmp_path):
    """16 sequences in four prompt groups (520, 700, 880 and 1000 ids); each group's four
    sequences differ in sampling parameters and seed, so their caches diverge from the first
    sampled id on.  The 1000-id group decodes past position 1024."""
    cfg = SMALL
    path = build_model_file(cfg, 7, tmp_path / "small.enargeia")
    f = read_enargeia(path)
    B, ctx, steps = 16, 1040, 30
    lengths = [520, 700, 880, 1000]
    rng = np.random.default_rng(4242)
    prompts = [[int(v) for v in rng.integers(0, cfg.vocab, L)] for L in lengths]
    plist = [GREEDY, APP_SAMPLING, SamplingParams(1.0, 1.0, 1.0), SamplingParams(0.5, 0.8, 1.3)]
    m = Model(cfg).load(path).kv_alloc(ctx, B)
    seqs = []
    for g, prompt in enumerate(prompts):
        base = oracle.OracleModel(f, cfg, ctx)
        ol0 = base.prefill(prompt, 256)
        for j in range(4):
            b = 4 * g + j
            p = plist[j]
            om = base if j == 3 else base.fork()
            os_ = oracle.OracleSession(om, p.temperature, p.top_p, p.repetition_penalty, seed=500 + b)
            draw = mulberry32(500 + b)
            m.prefill(b, prompt, 256)
            within(m.logits(b), ol0)
            os_.tokens = list(prompt)
            want = os_._sample(ol0.copy())
            got = m.sample_prefill(b, p, float(np.float32(draw())))
            assert got == want, (b, got, want)
            os_.tokens.append(want)
            seqs.append((p, om, os_, draw))
    toks = [s[2].tokens[-1] for s in seqs]
    params = [s[0] for s in seqs]
    for step in range(steps):
        randoms = [float(np.float32(s[3]())) for s in seqs]
        got = m.decode_step(toks, params, randoms)
        for b, (p, om, os_, draw) in enumerate(seqs):
            olp = om.decode(toks[b]).copy()
            want = os_._sample(olp)
            within(m.logits(b), olp)
            assert got[b] == want, (step, b, got[b], want)
            os_.tokens.append(want)
        toks = got
    assert seqs[-1][1].filled > 1024
    _check_cache(m, seqs[-1][1], cfg.layers, seqs[-1][1].filled, cfg.kv_dim, seq=B - 1)
    m.close()
