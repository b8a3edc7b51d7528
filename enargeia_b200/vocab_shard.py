"""Vocab-sharded tied LM head with sampling across GPUs.

The reference runs the tied int8 head and the sampler over the whole 151,936-id vocabulary on
one device (src/kernels/embedding_variants.ts:135-180 for the head, src/kernels/sample.wgsl:143-332
for the sampler, driven from src/model/graph.ts).  Here rank r of `world` holds the contiguous
row range `shard_range(vocab, world, r)` of the table, computes its slice of the logits, and the
ranks run the sampler's phases on their slices with a small allgather between phases (the
exchange the C ABI's enx_shard_* entry points define):

    prepare -> cand  -> probs -> sum -> buckets x4 (top-p) -> kept -> pick -> finish

The protocol is a generator (`ShardedSampler.protocol`) that yields each send buffer and
receives the gathered [world * len] buffer back, so the same sequence of phases runs

  * over torch.distributed (`run_distributed`: NCCL all_gather_into_tensor between GPUs, gloo
    all_gather on CPU),
  * or for several shards in one process (`run_lockstep`), which gathers by concatenation.

Every rank ends with the same ids.  The phases are pluggable: `CudaPhases` (libenx, the product
path) or any object with the same methods.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import EmbeddingDims, SamplingRow, call

ROUNDS = 4  # top-p bisection rounds of 8 steps (32 steps, sample.wgsl's loop count)


def shard_range(vocab: int, world: int, rank: int) -> Tuple[int, int]:
    """(row_begin, rows) of rank's contiguous id range: equal even-sized ranges, the last one
    shorter, so every range starts on an even row (the int8 table's packed zero-points hold 4
    blocks per word and a 896-wide row has 14 blocks)."""
    if not 0 <= rank < world:
        raise ValueError("rank outside world")
    per = -(-vocab // world)
    per += per & 1
    begin = min(rank * per, vocab)
    return begin, min(begin + per, vocab) - begin


def shard_rows(t, begin: int, count: int):
    """Rows [begin, begin + count) of a quantised table as its own (packed, scales, zeros)
    arrays in the .enargeia layout (zero-points repacked from block index 0)."""
    bits = t.bits
    per_word = 32 // bits
    words_per_row = t.cols * bits // 32
    bpr = t.cols // 64
    packed = np.ascontiguousarray(t.packed[begin * words_per_row:(begin + count) * words_per_row])
    scales = np.ascontiguousarray(t.scales[begin * bpr:(begin + count) * bpr])
    nblk = t.rows * bpr
    shifts = np.arange(per_word, dtype=np.uint32) * np.uint32(bits)
    codes = ((t.zeros[:, None] >> shifts[None, :]) & np.uint32((1 << bits) - 1)).reshape(-1)[:nblk]
    mine = codes[begin * bpr:(begin + count) * bpr]
    pad = np.zeros(-(-mine.size // per_word) * per_word, np.uint32)
    pad[:mine.size] = mine
    zeros = np.zeros(pad.size // per_word, np.uint32)
    for j in range(per_word):
        zeros |= pad.reshape(-1, per_word)[:, j] << shifts[j]
    return packed, scales, zeros


def default_split(rows: int, n: int, sms: int = 148) -> int:
    """CTAs per row and shard: enough to cover the SMs at small batch, at least ~2k ids each."""
    by_sms = max(1, sms // max(rows, 1))
    by_ids = max(1, n // 2048)
    return int(max(1, min(32, by_sms, by_ids)))


def sampling_rows_tensor(params: Sequence[Tuple[float, float, float, float]], device) -> torch.Tensor:
    arr = (SamplingRow * len(params))(*[SamplingRow(*map(float, p)) for p in params])
    return torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(device)


def _p(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


class CudaPhases:
    """The device phases: libenx's enx_shard_* kernels on `stream` (default: torch's current)."""

    def __init__(self, stream: Optional[torch.cuda.Stream] = None):
        self.stream = stream

    def _s(self):
        s = self.stream if self.stream is not None else torch.cuda.current_stream()
        return C.c_void_p(s.cuda_stream)

    def state(self, rows: int, device) -> torch.Tensor:
        return torch.zeros(int(_lib.load().enx_shard_state_bytes(rows)), dtype=torch.uint8, device=device)

    def prepare(self, logits, n, row_begin, rows, split, history, hstride, hist_len, params, cand):
        call("enx_shard_prepare", _p(logits), n, row_begin, rows, split, _p(history), hstride, _p(hist_len),
             _p(params), _p(cand), self._s())

    def probs(self, logits, n, rows, split, world, params, cand_all, state, probs, sums):
        call("enx_shard_probs", _p(logits), n, rows, split, world, _p(params), _p(cand_all), _p(state), _p(probs),
             _p(sums), self._s())

    def buckets(self, n, rows, split, world, rnd, params, sum_all, prev, state, probs, bucket):
        call("enx_shard_buckets", n, rows, split, world, rnd, _p(params), _p(sum_all), _p(prev), _p(state),
             _p(probs), _p(bucket), self._s())

    def kept(self, n, rows, split, world, rounds, params, sum_all, last, state, probs, kept):
        call("enx_shard_kept", n, rows, split, world, rounds, _p(params), _p(sum_all), _p(last), _p(state),
             _p(probs), _p(kept), self._s())

    def pick(self, n, row_begin, rows, split, world, rank, params, kept_all, state, probs, pick):
        call("enx_shard_pick", n, row_begin, rows, split, world, rank, _p(params), _p(kept_all), _p(state),
             _p(probs), _p(pick), self._s())

    def finish(self, rows, split, world, params, cand_all, pick_all, state, out):
        call("enx_shard_finish", rows, split, world, _p(params), _p(cand_all), _p(pick_all), _p(state), _p(out),
             self._s())


@dataclass
class ShardInputs:
    logits: torch.Tensor          # f32 [rows, n], penalised in place
    history: Optional[torch.Tensor]  # u32 bits in int32 [rows, stride]
    history_length: Optional[torch.Tensor]  # int32 [rows]
    params: Sequence[Tuple[float, float, float, float]]  # (temperature, top_p, penalty, random)


class ShardedSampler:
    """One rank's half of the sharded sampler: buffers for `rows` rows of an `n`-id shard."""

    def __init__(self, vocab: int, rank: int, world: int, rows: int, device, split: Optional[int] = None,
                 phases=None):
        self.vocab, self.rank, self.world, self.rows = vocab, rank, world, rows
        self.row_begin, self.n = shard_range(vocab, world, rank)
        if self.n == 0:
            raise ValueError("empty shard: more ranks than ids")
        self.device = torch.device(device)
        self.split = split or default_split(rows, self.n)
        self.ph = phases if phases is not None else CudaPhases()
        R, S, dev = rows, self.split, self.device
        self.state = self.ph.state(R, dev)
        self.probs = torch.empty(R * self.n, dtype=torch.float64, device=dev)
        self.cand = torch.empty(R * S * 4, dtype=torch.int32, device=dev)
        self.sums = torch.empty(R * S, dtype=torch.float64, device=dev)
        self.bucket = torch.empty(R * S * 256, dtype=torch.int64, device=dev)  # u64 fixed-point masses
        self.kept_buf = torch.empty(R * S, dtype=torch.float64, device=dev)
        self.pick_buf = torch.empty(R * S, dtype=torch.int32, device=dev)
        self.out = torch.empty(R, dtype=torch.int32, device=dev)

    def max_record_bytes(self) -> int:
        """The largest record one rank sends in one exchange (the top-p bucket masses)."""
        R, S = self.rows, self.split
        return max(R * S * 4 * 4, R * S * 8, R * S * 256 * 8, R * S * 4)

    @staticmethod
    def rounds_for(params) -> int:
        return ROUNDS if any(p[0] > 0.0 and p[1] < 1.0 for p in params) else 0

    def protocol(self, x: ShardInputs, params_dev: Optional[torch.Tensor] = None):
        """Generator: yields each send buffer, expects the gathered buffer of all ranks back
        (rank-major), returns the ids [rows] (device int32) through StopIteration."""
        if x.logits.shape != (self.rows, self.n):
            raise ValueError(f"logits must be [{self.rows}, {self.n}]")
        if len(x.params) != self.rows:
            raise ValueError("one sampling row per logits row")
        R, S, W, n, ph = self.rows, self.split, self.world, self.n, self.ph
        pr = params_dev if params_dev is not None else sampling_rows_tensor(x.params, self.device)
        hstride = 0 if x.history is None else int(x.history.shape[1])
        ph.prepare(x.logits, n, self.row_begin, R, S, x.history, hstride, x.history_length, pr, self.cand)
        cand_all = yield self.cand
        ph.probs(x.logits, n, R, S, W, pr, cand_all, self.state, self.probs, self.sums)
        sum_all = yield self.sums
        rounds = self.rounds_for(x.params)
        prev = None
        for r in range(rounds):
            ph.buckets(n, R, S, W, r, pr, sum_all, prev, self.state, self.probs, self.bucket)
            prev = yield self.bucket
        ph.kept(n, R, S, W, rounds, pr, sum_all, prev, self.state, self.probs, self.kept_buf)
        kept_all = yield self.kept_buf
        ph.pick(n, self.row_begin, R, S, W, self.rank, pr, kept_all, self.state, self.probs, self.pick_buf)
        pick_all = yield self.pick_buf
        ph.finish(R, S, W, pr, cand_all, pick_all, self.state, self.out)
        return self.out


def torch_allgather(group=None) -> Callable[[torch.Tensor], torch.Tensor]:
    """Rank-major allgather over torch.distributed: all_gather_into_tensor on NCCL, a list
    all_gather + cat elsewhere (gloo)."""
    import torch.distributed as dist

    nccl = dist.get_backend(group) == "nccl"
    world = dist.get_world_size(group)

    def gather(t: torch.Tensor) -> torch.Tensor:
        if nccl:
            out = torch.empty(world * t.numel(), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(out, t, group=group)
            return out
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t, group=group)
        return torch.cat(parts)

    return gather


class _DeviceView:
    """A raw device range as a torch tensor (zero copy, __cuda_array_interface__)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerGather:
    """Rank-major all-gather over peer memory (enx_peer_allgather): each rank stores its records
    straight into every other rank's exchange buffer over NVLink and raises an arrival word; one
    launch per exchange, no collective library.  Drop-in for torch_allgather in run_distributed.

    Each exchange lands in its own region of a ring of `regions`: the protocol reads a phase's
    gathered records again several phases later (the candidates in `finish`), so a region must not
    be overwritten by the next step's exchanges while it can still be read; 16 regions leave a
    whole step of margin over the 8 exchanges of a top-p step.  `max_bytes`: the largest record of
    one rank in one exchange."""

    def __init__(self, max_bytes: int, group=None, regions: int = 16, stream=None):
        import torch.distributed as dist

        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.region = -(-max_bytes // 16) * 16 * self.world
        self.regions = regions
        self.stream = stream
        own = C.c_void_p()
        handle = (C.c_uint8 * 64)()
        call("enx_peer_alloc", self.region * regions, C.byref(own), handle)
        self.own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.mapped = []
        addrs = []
        for p, hb in enumerate(handles):
            if p == self.rank:
                addrs.append(self.own)
                continue
            ptr = C.c_void_p()
            call("enx_peer_open", (C.c_uint8 * 64).from_buffer_copy(hb), C.byref(ptr))
            self.mapped.append(ptr.value)
            addrs.append(ptr.value)
        self.err = torch.zeros(1, dtype=torch.int32, device="cuda")
        # every region's world addresses, on the device once
        self.peer_tabs = [torch.tensor([a + r * self.region for a in addrs], dtype=torch.int64, device="cuda")
                          for r in range(regions)]
        self.seq = 0
        torch.cuda.synchronize()
        dist.barrier(group=group)  # every buffer mapped everywhere before the first exchange

    def __call__(self, t: torch.Tensor) -> torch.Tensor:
        t = t.contiguous()
        nb = t.numel() * t.element_size()
        padded = -(-nb // 16) * 16
        if padded * self.world > self.region:
            raise ValueError("record larger than the exchange region")
        src = t
        if padded != nb:
            src = torch.zeros(padded, dtype=torch.uint8, device=t.device)
            src[:nb].copy_(t.view(torch.uint8).reshape(-1))
        self.seq += 1
        r = self.seq % self.regions
        s = self.stream if self.stream is not None else torch.cuda.current_stream()
        call("enx_peer_allgather", C.c_void_p(src.data_ptr()), padded, C.c_void_p(self.peer_tabs[r].data_ptr()),
             self.world, self.rank, self.seq, C.c_void_p(self.err.data_ptr()), C.c_void_p(s.cuda_stream))
        self._keep = src  # alive until the launch has read it (same stream)
        raw = torch.as_tensor(_DeviceView(self.own + r * self.region + 512, padded * self.world), device=t.device)
        if padded != nb:
            raw = raw.view(self.world, padded)[:, :nb].contiguous().reshape(-1)
        return raw.view(t.dtype)

    def check(self) -> None:
        """Raise if an exchange's bounded wait gave up (a peer never arrived)."""
        if int(self.err.item()):
            raise _lib.EnxError(5, "peer exchange: a bounded wait for a peer's arrival gave up")

    def close(self) -> None:
        for p in self.mapped:
            _lib.load().enx_peer_close(C.c_void_p(p), 1)
        self.mapped = []
        if self.own:
            _lib.load().enx_peer_close(C.c_void_p(self.own), 0)
            self.own = None


def run_distributed(sampler: ShardedSampler, x: ShardInputs, gather: Optional[Callable] = None,
                    params_dev: Optional[torch.Tensor] = None) -> torch.Tensor:
    gather = gather or torch_allgather()
    gen = sampler.protocol(x, params_dev)
    send = next(gen)
    try:
        while True:
            send = gen.send(gather(send))
    except StopIteration as stop:
        return stop.value


def run_lockstep(samplers: Sequence[ShardedSampler], inputs: Sequence[ShardInputs]) -> List[torch.Tensor]:
    """All ranks of one vocabulary in one process (any devices): each phase runs on every rank,
    then the send buffers are concatenated in rank order and handed to every rank."""
    gens = [s.protocol(x) for s, x in zip(samplers, inputs)]
    sends = [next(g) for g in gens]
    while True:
        dev0 = sends[0].device
        gathered = torch.cat([s.to(dev0) for s in sends])
        nxt, done = [], None
        for s, g in zip(samplers, gens):
            try:
                nxt.append(g.send(gathered.to(s.device)))
            except StopIteration as stop:
                done = done or []
                done.append(stop.value)
        if done is not None:
            if len(done) != len(gens):
                raise RuntimeError("ranks left the protocol at different phases")
            return done
        sends = nxt


class ShardedHead:
    """Rank's rows of the tied int8 head on its GPU, and the logits of `rows` hidden states."""

    def __init__(self, table, vocab: int, rank: int, world: int, device):
        self.row_begin, self.n = shard_range(vocab, world, rank)
        self.hidden = table.cols
        packed, scales, zeros = shard_rows(table, self.row_begin, self.n)
        dev = torch.device(device)
        self.packed = torch.from_numpy(packed.view(np.int32)).to(dev)
        self.scales = torch.from_numpy(scales).to(dev)
        self.zeros = torch.from_numpy(zeros.view(np.int32)).to(dev)

    def logits(self, x: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
        """x f32 [rows, hidden] -> out f32 [rows, n] (enx_lm_head_q8 over this shard's rows)."""
        rows = x.shape[0]
        d = EmbeddingDims(rows, self.hidden, self.row_begin, self.n, 64, self.hidden // 64, self.n, 0,
                          min(self.n, 65535), 0, 0, 0)
        s = stream if stream is not None else torch.cuda.current_stream()
        call("enx_lm_head_q8", _p(x), _p(self.packed), _p(self.scales), _p(self.zeros), _p(out), C.byref(d),
             C.c_void_p(s.cuda_stream))
        return out
