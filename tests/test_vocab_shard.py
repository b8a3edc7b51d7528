"""Host logic of the vocab-sharded head and sampler (enargeia_b200/vocab_shard.py) on CPU: shard
ranges and table slicing, and the phase protocol - driven in lockstep in one process and across
two gloo ranks - against the CPU oracle's unsharded sampler (test/reference sampling semantics,
src/kernels/sample.wgsl:143-332).  The device phases are replaced by a numpy twin with the same
buffers; the CUDA phases themselves are checked in test_gpu_vocab_shard.py."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from enargeia_b200.format import quantize_tensor
from enargeia_b200.vocab_shard import (ShardedSampler, ShardInputs, run_distributed, run_lockstep, shard_range,
                                       shard_rows, torch_allgather)
from shard_twin import NumpyPhases

PARAMS = [  # (temperature, top_p, repetition_penalty)
    (0.0, 1.0, 1.0), (0.7, 0.9, 1.1), (1.0, 1.0, 1.0), (0.5, 0.5, 1.3), (0.0, 1.0, 1.1), (1.2, 0.99, 1.0),
]


@pytest.mark.parametrize("vocab,world", [(151936, 8), (151936, 3), (10, 4), (7, 7), (1000, 1)])
def test_shard_ranges_cover_the_vocabulary_in_order(vocab, world):
    nxt = 0
    for r in range(world):
        b, n = shard_range(vocab, world, r)
        assert b == nxt or n == 0
        assert b % 2 == 0 or n == 0
        nxt = b + n
    assert nxt == vocab


def test_shard_rows_slice_the_table():
    rng = np.random.default_rng(3)
    t = quantize_tensor("embed", rng.standard_normal((150, 128)).astype(np.float32) * 0.02, 8)
    full = t.dequantize()
    for world in (1, 2, 4, 7):
        got = []
        for r in range(world):
            b, n = shard_range(150, world, r)
            packed, scales, zeros = shard_rows(t, b, n)
            sub = quantize_tensor("x", np.zeros((max(n, 1), 128), np.float32), 8)
            sub.shape = (n, 128)
            sub.packed, sub.scales, sub.zeros = packed, scales, zeros
            got.append(sub.dequantize() if n else np.zeros((0, 128), np.float32))
        np.testing.assert_array_equal(np.concatenate(got), full)


def make_case(vocab, rows, seed, hist=300):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    logits[0, vocab // 2] = logits[0].max()  # a tie across shards for the greedy row
    history = rng.integers(0, vocab, (rows, hist)).astype(np.uint32)
    hlen = rng.integers(0, hist + 1, rows).astype(np.int32)
    params = []
    for r in range(rows):
        T, tp, rp = PARAMS[r % len(PARAMS)]
        params.append((T, tp, rp, float(np.float32(rng.random()))))
    return logits, history, hlen, params


def oracle_ids(oracle, logits, history, hlen, params):
    out = []
    for r in range(logits.shape[0]):
        T, tp, rp, rnd = params[r]
        out.append(oracle.sample(logits[r].copy(), history[r, :hlen[r]], T, tp, rp, rnd))
    return out


def shard_inputs(logits, history, hlen, params, vocab, world, rank):
    b, n = shard_range(vocab, world, rank)
    return ShardInputs(torch.from_numpy(np.ascontiguousarray(logits[:, b:b + n])),
                       torch.from_numpy(history.view(np.int32)), torch.from_numpy(hlen), params)


@pytest.mark.parametrize("vocab,world,split", [(4000, 1, 3), (4000, 2, 1), (4000, 3, 4), (3001, 8, 2),
                                               (151936, 4, 2)])
def test_lockstep_protocol_matches_unsharded_oracle(oracle, vocab, world, split):
    rows = 6
    logits, history, hlen, params = make_case(vocab, rows, 40 + world)
    samplers = [ShardedSampler(vocab, r, world, rows, "cpu", split=split, phases=NumpyPhases()) for r in range(world)]
    inputs = [shard_inputs(logits, history, hlen, params, vocab, world, r) for r in range(world)]
    outs = run_lockstep(samplers, inputs)
    want = oracle_ids(oracle, logits, history, hlen, params)
    for o in outs:
        assert [int(v) for v in o.numpy().view(np.uint32)] == want


def test_lockstep_without_top_p_skips_the_bucket_rounds(oracle):
    vocab, world, rows = 2000, 2, 3
    logits, history, hlen, _ = make_case(vocab, rows, 77)
    params = [(0.8, 1.0, 1.1, 0.3), (0.0, 1.0, 1.0, 0.5), (2.0, 1.0, 1.0, 0.999)]
    assert ShardedSampler.rounds_for(params) == 0
    samplers = [ShardedSampler(vocab, r, world, rows, "cpu", split=2, phases=NumpyPhases()) for r in range(world)]
    outs = run_lockstep(samplers, [shard_inputs(logits, history, hlen, params, vocab, world, r) for r in range(world)])
    assert [int(v) for v in outs[0].numpy()] == oracle_ids(oracle, logits, history, hlen, params)


def _gloo_rank(rank, world, port, vocab, rows, seed, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        logits, history, hlen, params = make_case(vocab, rows, seed)
        s = ShardedSampler(vocab, rank, world, rows, "cpu", split=2, phases=NumpyPhases())
        ids = run_distributed(s, shard_inputs(logits, history, hlen, params, vocab, world, rank), torch_allgather())
        q.put((rank, [int(v) for v in ids.numpy().view(np.uint32)]))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_match_unsharded_oracle(oracle):
    vocab, rows, seed, world = 5000, 6, 91, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, vocab, rows, seed, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    logits, history, hlen, params = make_case(vocab, rows, seed)
    want = oracle_ids(oracle, logits, history, hlen, params)
    assert got[0] == want and got[1] == want
