"""torchrun worker for the multi-GPU vocab-sharded head test: every rank builds the same seeded
int8 table and hidden states, takes its contiguous row range, computes its logits slice with
enx_lm_head_q8 and samples through the NCCL phase exchange.  Rank 0 writes the ids (and each
rank's own ids, which must agree) to the JSON file given as argv[1].

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        tests/dist_vocab_shard.py out.json [peer]

With "peer" the phases exchange through enx_peer_allgather (NVLink peer stores) instead of NCCL.
"""

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from enargeia_b200.format import quantize_tensor  # noqa: E402
from enargeia_b200.vocab_shard import PeerGather, ShardedHead, ShardedSampler, ShardInputs, run_distributed  # noqa: E402

VOCAB, HIDDEN, ROWS, HIST = 151936, 896, 8, 2048


def case():
    rng = np.random.default_rng(5150)
    table = quantize_tensor("embed", (rng.standard_normal((VOCAB, HIDDEN), dtype=np.float32) * 0.02), 8)
    x = rng.standard_normal((ROWS, HIDDEN)).astype(np.float32)
    history = rng.integers(0, VOCAB, (ROWS, HIST)).astype(np.uint32)
    params = [(0.0, 1.0, 1.1, 0.5)] + [(0.7, 0.9, 1.1, float(np.float32(rng.random()))) for _ in range(ROWS - 1)]
    return table, x, history, params


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    table, x, history, params = case()
    head = ShardedHead(table, VOCAB, rank, world, dev)
    logits = torch.empty((ROWS, head.n), dtype=torch.float32, device=dev)
    head.logits(torch.from_numpy(x).to(dev), logits)
    s = ShardedSampler(VOCAB, rank, world, ROWS, dev)
    hist = torch.from_numpy(history.view(np.int32)).to(dev)
    hlen = torch.full((ROWS,), HIST, dtype=torch.int32, device=dev)
    logits0 = logits.clone()  # the sampler penalises in place
    gather = None
    if len(sys.argv) > 2 and sys.argv[2] == "peer":  # peer-memory exchange instead of NCCL
        gather = PeerGather(s.max_record_bytes())
    ids = run_distributed(s, ShardInputs(logits, hist, hlen, params), gather).clone()
    if gather is not None:
        torch.cuda.synchronize()
        gather.check()
        # a second step through the same buffers (the ring of exchange regions moves on)
        ids2 = run_distributed(s, ShardInputs(logits0, hist, hlen, params), gather)
        torch.cuda.synchronize()
        gather.check()
        assert torch.equal(ids, ids2), "second exchange step disagrees"
        gather.close()
    mine = [int(v) for v in ids.cpu().numpy().view(np.uint32)]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    if rank == 0:
        Path(sys.argv[1]).write_text(json.dumps({"world": world, "ids": gathered}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
