"""The raw kernel entry points of libenx, over torch CUDA tensors.

Each function mirrors one WGSL dispatch of the reference (inputs, output, dims) and calls the
C ABI directly.  torch is only the allocator and stream provider here.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib
from ._lib import AttnDecodeDims, EmbeddingDims, MatmulQ4Dims, SampleDims, SamplingRow, call


def _ptr(t: Optional[torch.Tensor]):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = torch.cuda.current_stream() if stream is None else stream
    return C.c_void_p(s.cuda_stream)


def _u32(t: torch.Tensor):
    # int32 storage reinterpreted as u32 on the device side
    if t.dtype not in (torch.int32, torch.uint32):
        raise ValueError("packed words must be int32/uint32 tensors")
    return _ptr(t)


def matmul_q4(x, packed, scales, zeros, bias, out, m, n, k, out_stride=None, out_offset=0, stream=None):
    """matmul_q4_decode / matmul_q4_prefill (src/kernels/matmul_q4.ts:50-64)."""
    d = MatmulQ4Dims(m, n, k, 1 if bias is not None else 0, 64, k // 64, n if out_stride is None else out_stride,
                     out_offset, min(n, 65535), 0, 0, 0)
    call("enx_matmul_q4", _ptr(x), _u32(packed), _ptr(scales), _u32(zeros), _ptr(bias), _ptr(out), C.byref(d),
         _stream(stream))
    return out


def set_wait_limit(spins: int, device: int = 0) -> None:
    """Polls a bounded device wait makes before it gives up (0: the default)."""
    call("enx_set_wait_limit", device, spins)


def raw_check():
    """Synchronise the device and raise if a bounded wait of the raw tensor-core GEMM gave up."""
    call("enx_raw_check")


def lm_head_q8(x, packed, scales, zeros, out, rows, hidden, row_begin=0, out_offset=0, stream=None):
    """lm_head_q8 (src/kernels/embedding_variants.ts:135-180)."""
    d = EmbeddingDims(1, hidden, row_begin, rows, 64, hidden // 64, 0, out_offset, min(rows, 65535), 0, 0, 0)
    call("enx_lm_head_q8", _ptr(x), _u32(packed), _ptr(scales), _u32(zeros), _ptr(out), C.byref(d), _stream(stream))
    return out


def embed_gather_q8(ids, packed, scales, zeros, out, hidden, row_begin, row_count, stream=None):
    """embed_gather_q8 (src/kernels/embedding_variants.ts:100-130)."""
    d = EmbeddingDims(ids.numel(), hidden, row_begin, row_count, 64, hidden // 64, 0, 0, 0, 0, 0, 0)
    call("enx_embed_gather_q8", _u32(ids), _u32(packed), _ptr(scales), _u32(zeros), _ptr(out), C.byref(d),
         _stream(stream))
    return out


def sample(logits, history, out, temperature, top_p, repetition_penalty, random, stream=None):
    """sample (src/kernels/sample.wgsl): in-place penalty on `logits`, one id to out[0]."""
    d = SampleDims(logits.numel(), 0 if history is None else history.numel(), temperature, top_p,
                   repetition_penalty, random, 0, 0)
    call("enx_sample", _ptr(logits), None if history is None or history.numel() == 0 else _u32(history), _u32(out),
         C.byref(d), None, _stream(stream))
    return out


def sample_batched(logits, history, history_length, rows, out, stream=None):
    """Rows of logits [B, V]; history [B, stride] (u32); history_length [B]; rows: a CUDA byte
    tensor of B SamplingRow structs (see `sampling_rows`)."""
    B, V = logits.shape
    call("enx_sample_batched", _ptr(logits), V, B, _u32(history), history.shape[1], _u32(history_length),
         _ptr(rows), _u32(out), _stream(stream))
    return out


def sampling_rows(params, device="cuda") -> torch.Tensor:
    """[(temperature, top_p, repetition_penalty, random), ...] -> device bytes of SamplingRow."""
    arr = (SamplingRow * len(params))(*[SamplingRow(*p) for p in params])
    host = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
    return host.to(device)


def attn_decode(q, k_cache, v_cache, out, position, heads, kv_heads, head_dim, workspace=None, stream=None):
    d = AttnDecodeDims(position, heads, kv_heads, head_dim, 0, kv_heads * head_dim, 0, 0)
    if workspace is None:
        n = _lib.load().enx_attn_decode_workspace_bytes(position + 1, heads, head_dim)
        workspace = torch.empty(n, dtype=torch.uint8, device=q.device)
    call("enx_attn_decode", _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), C.byref(d), _ptr(workspace),
         _stream(stream))
    return out


def attn_prefill(q, k_cache, v_cache, out, queries, begin, heads, kv_heads, head_dim, workspace=None, stream=None):
    if workspace is None:
        n = _lib.load().enx_attn_prefill_workspace_bytes(queries, begin + queries, heads, head_dim)
        workspace = torch.empty(n, dtype=torch.uint8, device=q.device)
    call("enx_attn_prefill", _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), queries, begin, heads, kv_heads,
         head_dim, _ptr(workspace), _stream(stream))
    return out


def rmsnorm(x, w, out, seq, features, eps=1e-6, stream=None):
    call("enx_rmsnorm", _ptr(x), _ptr(w), _ptr(out), seq, features, eps, _stream(stream))
    return out


def rope(x, out, cos_t, sin_t, seq, heads, head_dim, pos0=0, out_offset=0, stream=None):
    call("enx_rope", _ptr(x), _ptr(out), _ptr(cos_t), _ptr(sin_t), seq, heads, head_dim, pos0, out_offset,
         _stream(stream))
    return out


def cache_pack(src, dst, count, dst_offset=0, stream=None):
    call("enx_cache_pack", _ptr(src), _ptr(dst), count, dst_offset, _stream(stream))
    return dst


def silu_mul(g, u, out, stream=None):
    call("enx_silu_mul", _ptr(g), _ptr(u), _ptr(out), g.numel(), _stream(stream))
    return out


def add(a, b, out, stream=None):
    call("enx_add", _ptr(a), _ptr(b), _ptr(out), a.numel(), _stream(stream))
    return out


def to_device_u32(a) -> torch.Tensor:
    """numpy uint32 -> CUDA int32 tensor with the same bits."""
    import numpy as np

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).cuda()
