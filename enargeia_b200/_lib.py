"""ctypes binding of libenx.so (include/enx.h).

There is no fallback: if the library is missing or fails to load, every call raises.  Build it
with `python -m enargeia_b200.build`.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libenx.so"

ENX_OK = 0
STATUS_NAMES = {1: "INVALID", 2: "CUDA", 3: "RANGE", 4: "FORMAT", 5: "TIMEOUT", 6: "NOMEM", 7: "STATE"}


class EnxError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{STATUS_NAMES.get(status, status)}] {message}")
        self.status = status


class EnxRangeError(EnxError, IndexError):
    """RangeError of the reference: context exhausted, prompt too long, grid limits."""


class EnargeiaFormatError(EnxError, ValueError):
    """EnargeiaError of the reference (src/model/enargeia.ts:68-74)."""


P = C.c_void_p
U32 = C.c_uint32
F32 = C.c_float


class MatmulQ4Dims(C.Structure):
    _fields_ = [(n, U32) for n in ("m", "n", "k", "use_bias", "block_size", "blocks_per_row", "out_stride",
                                   "out_offset", "grid_width", "pad0", "pad1", "pad2")]


class EmbeddingDims(C.Structure):
    _fields_ = [(n, U32) for n in ("seq", "hidden", "row_begin", "row_count", "block_size", "blocks_per_row",
                                   "out_stride", "out_offset", "grid_width", "pad0", "pad1", "pad2")]


class SampleDims(C.Structure):
    _fields_ = [("vocab", U32), ("history_length", U32), ("temperature", F32), ("top_p", F32),
                ("repetition_penalty", F32), ("random", F32), ("pad0", U32), ("pad1", U32)]


class SamplingRow(C.Structure):
    _fields_ = [("temperature", F32), ("top_p", F32), ("repetition_penalty", F32), ("random", F32)]


class AttnDecodeDims(C.Structure):
    _fields_ = [(n, U32) for n in ("position", "heads", "kv_heads", "head_dim", "score_stride", "cache_stride",
                                   "pad0", "pad1")]


class ModelConfigC(C.Structure):
    _fields_ = [("layers", U32), ("hidden", U32), ("heads", U32), ("kv_heads", U32), ("head_dim", U32),
                ("intermediate", U32), ("vocab", U32), ("rms_norm_eps", F32), ("rope_theta", F32)]


class SamplingC(C.Structure):
    _fields_ = [("temperature", F32), ("top_p", F32), ("repetition_penalty", F32)]


assert C.sizeof(MatmulQ4Dims) == 48 and C.sizeof(EmbeddingDims) == 48
assert C.sizeof(SampleDims) == 32 and C.sizeof(AttnDecodeDims) == 32

# name -> (restype, argtypes)
SIGNATURES = {
    "enx_last_error": (C.c_char_p, []),
    "enx_version": (C.c_char_p, []),
    "enx_matmul_q4": (C.c_int32, [P, P, P, P, P, P, C.POINTER(MatmulQ4Dims), P]),
    "enx_set_wait_limit": (C.c_int32, [C.c_int, U32]),
    "enx_nll": (C.c_int32, [P, U32, U32, C.POINTER(C.c_double)]),
    "enx_peer_alloc": (C.c_int32, [C.c_size_t, C.POINTER(P), P]),
    "enx_peer_open": (C.c_int32, [P, C.POINTER(P)]),
    "enx_peer_close": (C.c_int32, [P, C.c_int]),
    "enx_peer_allgather": (C.c_int32, [P, C.c_size_t, P, U32, U32, C.c_uint64, P, P]),
    "enx_lm_head_q8": (C.c_int32, [P, P, P, P, P, C.POINTER(EmbeddingDims), P]),
    "enx_embed_gather_q8": (C.c_int32, [P, P, P, P, P, C.POINTER(EmbeddingDims), P]),
    "enx_sample": (C.c_int32, [P, P, P, C.POINTER(SampleDims), P, P]),
    "enx_sample_batched": (C.c_int32, [P, U32, U32, P, U32, P, P, P, P]),
    "enx_attn_decode": (C.c_int32, [P, P, P, P, C.POINTER(AttnDecodeDims), P, P]),
    "enx_attn_decode_noalloc": (C.c_int32, [P, P, P, P, C.POINTER(AttnDecodeDims), P]),
    "enx_attn_decode_workspace_bytes": (C.c_size_t, [U32, U32, U32]),
    "enx_attn_prefill": (C.c_int32, [P, P, P, P, U32, U32, U32, U32, U32, P, P]),
    "enx_attn_prefill_workspace_bytes": (C.c_size_t, [U32, U32, U32, U32]),
    "enx_rmsnorm": (C.c_int32, [P, P, P, U32, U32, F32, P]),
    "enx_rope": (C.c_int32, [P, P, P, P, U32, U32, U32, U32, U32, P]),
    "enx_cache_pack": (C.c_int32, [P, P, U32, U32, P]),
    "enx_silu_mul": (C.c_int32, [P, P, P, U32, P]),
    "enx_add": (C.c_int32, [P, P, P, U32, P]),
    "enx_create": (C.c_int32, [C.POINTER(ModelConfigC), C.c_int, C.POINTER(P)]),
    "enx_destroy": (C.c_int32, [P]),
    "enx_load_enargeia": (C.c_int32, [P, C.c_char_p]),
    "enx_load_enargeia_memory": (C.c_int32, [P, P, C.c_size_t]),
    "enx_kv_alloc": (C.c_int32, [P, U32, U32]),
    "enx_kv_reset": (C.c_int32, [P, U32]),
    "enx_kv_filled": (C.c_int32, [P, U32, C.POINTER(U32)]),
    "enx_raw_check": (C.c_int32, []),
    "enx_prefill": (C.c_int32, [P, U32, P, U32, U32]),
    "enx_sample_prefill": (C.c_int32, [P, U32, C.POINTER(SamplingC), F32, C.POINTER(U32)]),
    "enx_decode_step": (C.c_int32, [P, U32, P, C.POINTER(SamplingC), U32, P, P]),
    "enx_decode_loop": (C.c_int32, [P, U32, P, C.POINTER(SamplingC), U32, U32, P, P, C.c_int]),
    "enx_synchronize": (C.c_int32, [P]),
    "enx_loop_ids": (C.c_int32, [P, P, U32]),
    "enx_logits": (C.c_int32, [P, U32, P]),
    "enx_hidden": (C.c_int32, [P, U32, P]),
    "enx_kv_view": (C.c_int32, [P, U32, U32, C.POINTER(P), C.POINTER(P)]),
    "enx_tensor_view": (C.c_int32, [P, C.c_char_p, C.POINTER(C.c_int32), C.POINTER(U32), C.POINTER(U32),
                                    C.POINTER(P), C.POINTER(P), C.POINTER(P)]),
    "enx_set_tracing": (C.c_int32, [P, C.c_int]),
    "enx_trace": (C.c_int32, [P, P, U32, C.POINTER(U32)]),
    "enx_stream": (C.c_int32, [P, C.POINTER(P)]),
    "enx_step_launches": (C.c_int32, [P, C.POINTER(U32)]),
    "enx_launch_step_kernel": (C.c_int32, [P, U32, U32]),
    "enx_batch_profile": (C.c_int32, [P, U32, C.POINTER(C.c_float), U32]),
    "enx_shard_state_bytes": (C.c_size_t, [U32]),
    "enx_shard_prepare": (C.c_int32, [P, U32, U32, U32, U32, P, U32, P, P, P, P]),
    "enx_shard_probs": (C.c_int32, [P, U32, U32, U32, U32, P, P, P, P, P, P]),
    "enx_shard_buckets": (C.c_int32, [U32, U32, U32, U32, U32, P, P, P, P, P, P, P]),
    "enx_shard_kept": (C.c_int32, [U32, U32, U32, U32, U32, P, P, P, P, P, P, P]),
    "enx_shard_pick": (C.c_int32, [U32, U32, U32, U32, U32, U32, P, P, P, P, P, P]),
    "enx_shard_finish": (C.c_int32, [U32, U32, U32, P, P, P, P, P, P]),
}

_lib = None


def load() -> C.CDLL:
    """Load libenx.so (raises if it is not built: there is no CPU fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m enargeia_b200.build`")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int) -> None:
    if status == ENX_OK:
        return
    msg = load().enx_last_error().decode(errors="replace")
    if status == 3:
        raise EnxRangeError(status, msg)
    if status == 4:
        raise EnargeiaFormatError(status, msg)
    raise EnxError(status, msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
