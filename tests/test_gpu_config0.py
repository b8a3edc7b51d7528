"""Config 0 at full size: the Qwen2.5-0.5B-architecture model (24 layers, vocab 151936, int4 +
int8 tied head, seeded random-init weights), a 32-id prompt decoded to 64 tokens, through the
public Session API on the GPU, against the CPU oracle.  Ids must be identical; logits within
1e-3 rel / 1e-4 abs and bit-identical except for rare last-bit ties."""

import os
from pathlib import Path

import numpy as np
import pytest

from enargeia_b200.checkpoint import QWEN2_0_5B, build_model_file
from enargeia_b200.format import read_enargeia
from enargeia_b200.session import APP_SAMPLING, GREEDY, Model, Session

pytestmark = pytest.mark.gpu

SEED = 20251201  # the bench model
MODEL = Path(os.environ.get("ENX_MODEL_DIR", "/tmp/enx_models")) / f"qwen2.5-0.5b-random-s{SEED}-q4q8.enargeia"


@pytest.fixture(scope="module")
def full():
    path = build_model_file(QWEN2_0_5B, SEED, MODEL)
    return path, read_enargeia(path)


def _check(m, om_logits):
    g = m.logits()
    err = np.abs(g.astype(np.float64) - om_logits)
    ratio = err / (1e-4 + 1e-3 * np.abs(om_logits))
    assert ratio.max() <= 1.0, float(ratio.max())
    assert np.mean(g == om_logits) >= 0.999, float(np.mean(g == om_logits))


@pytest.mark.parametrize("params,seed,n", [(GREEDY, 1, 64), (APP_SAMPLING, 0x5EED, 32)])
def test_config0_session_matches_oracle(gpu, oracle, full, params, seed, n):
    path, f = full
    prompt = [int(v) for v in np.random.default_rng(1000).integers(0, QWEN2_0_5B.vocab, 32)]
    ctx = 32 + n + 1
    m = Model(QWEN2_0_5B).load(path).kv_alloc(ctx)
    s = Session(m, params, seed=seed)
    om = oracle.OracleModel(f, QWEN2_0_5B, ctx)
    os_ = oracle.OracleSession(om, params.temperature, params.top_p, params.repetition_penalty, seed)
    s.prime(prompt)
    ol = om.prefill(prompt)
    _check(m, ol)
    os_.tokens = list(prompt)
    want = os_._sample(ol.copy())
    got = s.sample_from_prefill()
    assert got == want
    s.tokens.append(got)
    os_.tokens.append(want)
    tok = got
    for step in range(1, n):
        ol = om.decode(tok)
        got = s.decode_step(tok)
        olp = ol.copy()
        want = os_._sample(olp)
        _check(m, olp)
        assert got == want, (step, got, want, os_.traces[-1])
        s.tokens.append(got)
        os_.tokens.append(want)
        tok = got
    m.close()
