"""enx_attn_decode_noalloc: the attention entry point for callers that cannot allocate device
memory (it keeps its split partials in a library-owned device array instead of a workspace).

Checked through the C ABI against enx_attn_decode (caller workspace) on two calls in a row, so a
second call that reuses the shared array must still be right.  This file sorts last so a run that
stops at the first failure has run everything else first."""

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-5, 1e-4  # same tolerance as the attention tests in test_gpu_kernels.py


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _case(position, seed, heads=14, kvh=2, hd=64):
    rng = np.random.default_rng(seed)
    n = position + 1
    q = torch.from_numpy(rng.standard_normal(heads * hd).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal(n * kvh * hd).astype(np.float16).view(np.int16)).cuda()
    v = torch.from_numpy(rng.standard_normal(n * kvh * hd).astype(np.float16).view(np.int16)).cuda()
    return q, k, v


def test_noalloc_matches_workspace_path_twice(gpu, oracle):
    from enargeia_b200 import _lib
    from enargeia_b200._lib import AttnDecodeDims

    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    heads, kvh, hd = 14, 2, 64
    for call, (position, seed) in enumerate([(700, 1), (95, 2)]):  # the second call reuses the array
        q, k, v = _case(position, seed)
        d = AttnDecodeDims(position, heads, kvh, hd, 0, kvh * hd, 0, 0)
        ws = torch.empty(lib.enx_attn_decode_workspace_bytes(position + 1, heads, hd), dtype=torch.uint8, device="cuda")
        ref = torch.zeros(heads * hd, dtype=torch.float32, device="cuda")
        got = torch.full((heads * hd,), float("nan"), dtype=torch.float32, device="cuda")
        _lib.check(lib.enx_attn_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(ref), C.byref(d), _ptr(ws), stream))
        _lib.check(lib.enx_attn_decode_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(got), C.byref(d), stream))
        torch.cuda.synchronize()
        a, b = got.cpu().numpy().astype(np.float64), ref.cpu().numpy().astype(np.float64)
        ratio = np.abs(a - b) / (ATOL + RTOL * np.abs(b))
        assert np.isfinite(a).all() and ratio.max() <= 1.0, (call, float(ratio.max()))
        # and independently against the CPU restatement of the reference's attention
        kb = k.cpu().numpy().view(np.uint16)
        vb = v.cpu().numpy().view(np.uint16)
        want = oracle.attention_f16(q.cpu().numpy(), kb, vb, position, heads, kvh, hd).reshape(-1).astype(np.float64)
        ratio = np.abs(a - want) / (ATOL + RTOL * np.abs(want))
        assert ratio.max() <= 1.0, (call, "oracle", float(ratio.max()))


def test_noalloc_rejects_oversize(gpu):
    from enargeia_b200 import _lib
    from enargeia_b200._lib import AttnDecodeDims

    lib = _lib.load()
    q, k, v = _case(3, 3)
    out = torch.zeros(14 * 64, dtype=torch.float32, device="cuda")
    d = AttnDecodeDims(4096, 14, 2, 64, 0, 128, 0, 0)
    st = lib.enx_attn_decode_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(out), C.byref(d), None)
    assert st == 3 and b"4096" in lib.enx_last_error()
