"""Model context and decode session over libenx: the host-side mirror of the reference runtime.

`Model` is WeightStore + KVCache ownership (src/model/weights.ts, src/runtime/kvcache.ts);
`Session` keeps the API of src/runtime/session.ts: `generate`, `decode_step`, `logits_after`,
`prime`, `reset`, `set_sampling`, `context_length`, the mulberry32 RNG seeded 0x5eed by default,
one draw per sampled token (the first token comes from the prefill logits), stop tokens and the
GenerateTiming fields.  All device work is libenx's; there is no CPU path.
"""

from __future__ import annotations

import ctypes as C
import math
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import ModelConfigC, SamplingC, call
from .checkpoint import ModelConfig

DEFAULT_PREFILL_CHUNK = 256


@dataclass(frozen=True)
class SamplingParams:
    """SamplingParams (src/kernels/sample.ts:24-33)."""

    temperature: float = 0.0
    top_p: float = 1.0
    repetition_penalty: float = 1.0


GREEDY = SamplingParams()
#: The values the reference app ships (src/ui/engine.ts:256-262).
APP_SAMPLING = SamplingParams(0.7, 0.9, 1.1)


def mulberry32(seed: int) -> Callable[[], float]:
    """Seeded draws in [0, 1) (src/runtime/session.ts:75-83)."""
    state = [seed & 0xFFFFFFFF]

    def draw() -> float:
        s = (state[0] + 0x6D2B79F5) & 0xFFFFFFFF
        state[0] = s
        t = ((s ^ (s >> 15)) * (1 | s)) & 0xFFFFFFFF
        t = ((t + (((t ^ (t >> 7)) * (61 | t)) & 0xFFFFFFFF)) & 0xFFFFFFFF) ^ t
        return ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296.0

    return draw


class Model:
    """A libenx context on one CUDA device: weights plus preallocated f16 KV caches."""

    def __init__(self, config: ModelConfig, device: int = 0):
        self.config = config
        self.device = device
        lib = _lib.load()
        c = ModelConfigC(config.layers, config.hidden, config.heads, config.kv_heads, config.head_dim,
                         config.intermediate, config.vocab, config.rms_norm_eps, config.rope_theta)
        h = C.c_void_p()
        _lib.check(lib.enx_create(C.byref(c), device, C.byref(h)))
        self._h = h
        self.max_context = 0
        self.batch = 0

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().enx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load(self, path) -> "Model":
        call("enx_load_enargeia", self._h, str(Path(path)).encode())
        return self

    def load_bytes(self, data: bytes) -> "Model":
        buf = C.create_string_buffer(data, len(data))
        call("enx_load_enargeia_memory", self._h, buf, len(data))
        return self

    def kv_alloc(self, max_context: int, batch: int = 1) -> "Model":
        call("enx_kv_alloc", self._h, max_context, batch)
        self.max_context = max_context
        self.batch = batch
        return self

    def filled(self, seq: int = 0) -> int:
        v = C.c_uint32()
        call("enx_kv_filled", self._h, seq, C.byref(v))
        return v.value

    def reset(self, seq: int = 0) -> None:
        call("enx_kv_reset", self._h, seq)

    def prefill(self, seq: int, ids: Sequence[int], chunk: int = DEFAULT_PREFILL_CHUNK) -> None:
        a = np.ascontiguousarray(ids, dtype=np.uint32)
        call("enx_prefill", self._h, seq, a.ctypes.data, a.size, chunk)

    def sample_prefill(self, seq: int, params: SamplingParams, random: float) -> int:
        out = C.c_uint32()
        p = SamplingC(params.temperature, params.top_p, params.repetition_penalty)
        call("enx_sample_prefill", self._h, seq, C.byref(p), random, C.byref(out))
        return out.value

    def decode_step(self, tokens: Sequence[int], params: Sequence[SamplingParams], randoms: Sequence[float]) -> List[int]:
        b = len(tokens)
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        r = np.ascontiguousarray(randoms, dtype=np.float32)
        ps = (SamplingC * len(params))(*[SamplingC(p.temperature, p.top_p, p.repetition_penalty) for p in params])
        out = np.zeros(b, dtype=np.uint32)
        call("enx_decode_step", self._h, b, t.ctypes.data, ps, len(params), r.ctypes.data, out.ctypes.data)
        return [int(v) for v in out]

    def decode_loop(self, first_tokens: Sequence[int], params: Sequence[SamplingParams], randoms: np.ndarray,
                    steps: int, sync: bool = True) -> Optional[np.ndarray]:
        """`steps` device-fed decode steps (see enx_decode_loop); returns ids [steps, batch] when
        sync, else None (then call synchronize() and loop_ids())."""
        b = len(first_tokens)
        t = np.ascontiguousarray(first_tokens, dtype=np.uint32)
        r = np.ascontiguousarray(randoms, dtype=np.float32).reshape(-1)
        if r.size != steps * b:
            raise ValueError("randoms must hold steps*batch draws")
        ps = (SamplingC * len(params))(*[SamplingC(p.temperature, p.top_p, p.repetition_penalty) for p in params])
        out = np.zeros(steps * b, dtype=np.uint32) if sync else None
        call("enx_decode_loop", self._h, b, t.ctypes.data, ps, len(params), steps, r.ctypes.data,
             None if out is None else out.ctypes.data, 1 if sync else 0)
        return None if out is None else out.reshape(steps, b)

    def synchronize(self) -> None:
        call("enx_synchronize", self._h)

    def loop_ids(self, steps: int, batch: int = 1) -> np.ndarray:
        out = np.zeros(steps * batch, dtype=np.uint32)
        call("enx_loop_ids", self._h, out.ctypes.data, steps * batch)
        return out.reshape(steps, batch)

    def logits(self, seq: int = 0) -> np.ndarray:
        out = np.empty(self.config.vocab, dtype=np.float32)
        call("enx_logits", self._h, seq, out.ctypes.data)
        return out

    def nll(self, target: int, seq: int = 0) -> float:
        """-log softmax(current logits of `seq`)[target], computed on the device (enx_nll)."""
        out = C.c_double()
        call("enx_nll", self._h, seq, int(target), C.byref(out))
        return out.value

    def hidden(self, seq: int = 0) -> np.ndarray:
        out = np.empty(self.config.hidden, dtype=np.float32)
        call("enx_hidden", self._h, seq, out.ctypes.data)
        return out

    def kv_view(self, seq: int, layer: int):
        """Device pointers (ints) of one layer's K and V cache of a sequence."""
        k, v = C.c_void_p(), C.c_void_p()
        call("enx_kv_view", self._h, seq, layer, C.byref(k), C.byref(v))
        return k.value, v.value

    def tensor_view(self, name: str):
        bits, rows, cols = C.c_int32(), C.c_uint32(), C.c_uint32()
        p, s, z = C.c_void_p(), C.c_void_p(), C.c_void_p()
        call("enx_tensor_view", self._h, name.encode(), C.byref(bits), C.byref(rows), C.byref(cols), C.byref(p),
             C.byref(s), C.byref(z))
        return dict(bits=bits.value, rows=rows.value, cols=cols.value, packed=p.value, scales=s.value, zeros=z.value)

    def step_launches(self) -> int:
        v = C.c_uint32()
        call("enx_step_launches", self._h, C.byref(v))
        return v.value

    def set_tracing(self, on: bool) -> None:
        call("enx_set_tracing", self._h, 1 if on else 0)

    def stage_times(self) -> dict:
        """Per-stage device times (us) of the last traced step, summed over layers: how long each
        stage waited for its barrier+weights and how long it computed (kernel-group telemetry of
        src/runtime/telemetry.ts, at stage granularity; telemetry.parse_stage_trace)."""
        from .telemetry import parse_stage_trace, trace_words

        L = self.config.layers
        n = trace_words(L)
        buf = np.zeros(n, dtype=np.uint64)
        cnt = C.c_uint32()
        call("enx_trace", self._h, buf.ctypes.data, n, C.byref(cnt))
        return parse_stage_trace(buf, L)

    def stream_handle(self) -> int:
        s = C.c_void_p()
        call("enx_stream", self._h, C.byref(s))
        return s.value or 0


@dataclass
class GenerateTiming:
    """GenerateTiming (src/runtime/session.ts:59-67)."""

    ttft_seconds: float
    prefill_seconds: float
    inter_token_seconds: List[float] = field(default_factory=list)
    tokens_per_second: float = 0.0


@dataclass
class GenerateResult:
    tokens: List[int]
    timing: GenerateTiming


class Session:
    """One conversation on sequence `seq` of a Model (Session, src/runtime/session.ts:85-504)."""

    def __init__(self, model: Model, sampling: SamplingParams = GREEDY, seed: int = 0x5EED, seq: int = 0,
                 prefill_chunk: int = DEFAULT_PREFILL_CHUNK):
        if model.max_context == 0:
            raise RuntimeError("allocate the KV cache first (Model.kv_alloc)")
        self.model = model
        self.sampling = sampling
        self.random = mulberry32(seed)
        self.seq = seq
        self.tokens: List[int] = []
        self.prefill_chunk = min(prefill_chunk, model.max_context)

    @property
    def context_length(self) -> int:
        return self.model.filled(self.seq)

    @property
    def remaining(self) -> int:
        return self.model.max_context - self.context_length

    def set_sampling(self, params: SamplingParams) -> None:
        self.sampling = params

    def reset(self, seed: Optional[int] = None) -> None:
        """Drop the conversation without freeing anything."""
        self.model.reset(self.seq)
        self.tokens = []
        if seed is not None:
            self.random = mulberry32(seed)

    def _draw(self) -> float:
        # the draw travels as an f32 in the uniform block (src/kernels/sample.ts:43-48)
        return float(np.float32(self.random()))

    def prime(self, prompt: Sequence[int]) -> float:
        """Prefill without generating; returns seconds (Session.prime / runPrefill)."""
        if len(prompt) > self.remaining:
            raise _lib.EnxRangeError(3, f"prompt of {len(prompt)} exceeds the remaining context of {self.remaining}")
        t0 = time.perf_counter()
        self.model.prefill(self.seq, prompt, self.prefill_chunk)
        self.tokens = list(prompt)
        return time.perf_counter() - t0

    def sample_from_prefill(self) -> int:
        return self.model.sample_prefill(self.seq, self.sampling, self._draw())

    def decode_step(self, token: int) -> int:
        """Append `token` at the next position and sample what follows."""
        return self.model.decode_step([token], [self.sampling], [self._draw()])[0]

    def logits_after(self, token: int) -> np.ndarray:
        """Run one step for `token` and return the full logits (evaluation path; the reference
        runs it at penalty 1, so the in-place penalty is a no-op there)."""
        self.model.decode_step([token], [self.sampling], [self._draw()])
        self.tokens.append(token)
        return self.model.logits(self.seq)

    def perplexity(self, tokens: Sequence[int]) -> float:
        """exp(mean nll) of tokens[2:] given their prefixes, the reference's cached evaluation
        (test/parity/quality.test.ts:111-139): prime with tokens[0], then for each later position
        one decode step (logitsAfter) and the nll of the next token, read back as 8 bytes (enx_nll)
        rather than the whole logits row.  Resets the session first."""
        if len(tokens) < 3:
            raise ValueError("perplexity needs at least 3 tokens")
        self.reset()
        self.prime(tokens[:1])
        total, counted = 0.0, 0
        for i in range(1, len(tokens) - 1):
            self.model.decode_step([tokens[i]], [self.sampling], [self._draw()])
            self.tokens.append(tokens[i])
            total += self.model.nll(tokens[i + 1], self.seq)
            counted += 1
        return math.exp(total / counted)

    def generate(self, prompt: Sequence[int], max_tokens: int, stop_tokens: Sequence[int] = (),
                 on_token: Optional[Callable[[int, int], None]] = None,
                 should_stop: Optional[Callable[[], bool]] = None) -> GenerateResult:
        stop = set(stop_tokens)
        start = time.perf_counter()
        prefill_s = self.prime(prompt)
        nxt = self.sample_from_prefill()
        ttft = time.perf_counter() - start
        produced = [nxt]
        if on_token:
            on_token(nxt, 0)
        self.tokens.append(nxt)
        inter: List[float] = []
        i = 1
        while i < max_tokens and nxt not in stop:
            if self.remaining <= 0:
                break
            if should_stop and should_stop():
                break
            t0 = time.perf_counter()
            nxt = self.decode_step(nxt)
            inter.append(time.perf_counter() - t0)
            produced.append(nxt)
            if on_token:
                on_token(nxt, i)
            self.tokens.append(nxt)
            i += 1
        mean = sum(inter) / len(inter) if inter else ttft
        return GenerateResult(produced, GenerateTiming(ttft, prefill_s, inter, 1.0 / mean if mean > 0 else 0.0))
