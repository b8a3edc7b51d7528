"""The bounded device-side waits give up and report instead of hanging.

With the wait limit set to one poll (enx_set_wait_limit), the persistent decode kernel's grid
barriers and the tensor-core GEMM's pipeline waits run out almost at once: each call must return
ENX_ERR_TIMEOUT, nothing faults or hangs, and with the default limit restored the same context
computes the same results as before.  No wait is made to run out by an error in the GPU's memory
or by a trap: the only change is how long each wait may poll."""

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from enargeia_b200 import kernels as K
from enargeia_b200._lib import EnxError
from enargeia_b200.checkpoint import TINY
from enargeia_b200.format import quantize_tensor
from enargeia_b200.session import GREEDY, Model

pytestmark = pytest.mark.gpu

TIMEOUT = 5  # ENX_ERR_TIMEOUT


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_gemm_wait_gives_up_then_recovers(gpu, oracle):
    n, k, m = 4864, 896, 256
    x = oracle.random_floats(m * k, 51)
    t = quantize_tensor("w", oracle.random_floats(n * k, 52).reshape(n, k), 4)
    p, s, z = K.to_device_u32(t.packed), dev(t.scales), K.to_device_u32(t.zeros)
    out = torch.zeros(m * n, dtype=torch.float32, device="cuda")
    K.raw_check()  # nothing pending
    K.set_wait_limit(1)
    try:
        K.matmul_q4(dev(x), p, s, z, None, out, m, n, k)
        with pytest.raises(EnxError) as e:
            K.raw_check()
        assert e.value.status == TIMEOUT and "tensor-core" in str(e.value)
    finally:
        K.set_wait_limit(0)
    K.raw_check()  # the sticky word was cleared by the failing check
    out.zero_()
    K.matmul_q4(dev(x), p, s, z, None, out, m, n, k)
    K.raw_check()
    want = oracle.linear_q(t, x.reshape(m, k)).reshape(m, n)
    got = out.cpu().numpy().reshape(m, n)
    err = np.abs(got.astype(np.float64) - want) / (1e-4 + 1e-4 * np.abs(want))
    assert err.max() <= 1.0


def _greedy_run(m, prompt, steps):
    m.reset(0)
    m.prefill(0, prompt, 20)
    tok = int(np.argmax(m.logits()))
    ids = [tok]
    for _ in range(steps):
        tok = m.decode_step([tok], [GREEDY], [0.5])[0]
        ids.append(tok)
    return ids, m.logits().copy()


def test_decode_and_prefill_waits_give_up_then_recover(gpu, oracle, tiny_file):
    prompt = [int(v) for v in np.random.default_rng(77).integers(0, TINY.vocab, 40)]
    m = Model(TINY).load(GOLDEN / "tiny_q8.enargeia").kv_alloc(64)
    base_ids, base_logits = _greedy_run(m, prompt, 6)
    m.reset(0)
    m.prefill(0, prompt[:8], 8)  # below 16 rows: no tensor-core wait in this prefill
    assert m.filled(0) == 8
    K.set_wait_limit(1)
    try:
        # the persistent step's grid barriers give up: the fill does not advance
        with pytest.raises(EnxError) as e:
            m.decode_step([prompt[8]], [GREEDY], [0.5])
        assert e.value.status == TIMEOUT and "enx_decode_step" in str(e.value)
        assert m.filled(0) == 8
        # a prefill chunk of 32 rows runs its projections on the tensor-core GEMM
        with pytest.raises(EnxError) as e:
            m.prefill(0, prompt[8:40], 32)
        assert e.value.status == TIMEOUT and "enx_prefill" in str(e.value)
        assert m.filled(0) == 8  # the fill from before the call
    finally:
        K.set_wait_limit(0)
    ids, logits = _greedy_run(m, prompt, 6)
    assert ids == base_ids
    np.testing.assert_array_equal(logits, base_logits)
    m.close()
