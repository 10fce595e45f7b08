"""One rank of the multi-GPU row-sharded decode check (launched by
tests/test_sharded_multi_gpu.py through torch.distributed.run).

Each rank holds its row slices of a two-layer stack (hidden 512, 4 query /
2 kv heads, FFN 768, vocab 512), runs ShardedDecode with the device kernels
and both all-gathers (NCCL, and the peer-memory kernel) for six positions at
batch 1 and batch 3 (batch 1 also with the RMSNorms inside the projections and
the residual gathered in place), and checks the
gathered logits against the unsharded float64 restatement
(||d||_inf / ||ref||_inf <= 2e-3). Exits non-zero on a mismatch.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main() -> int:
    import torch
    import torch.distributed as dist

    from cybel_b200.decode import StackShape, random_layer, random_rows
    from cybel_b200.formats import Q4_K, Q6_K
    from cybel_b200.sharded import GpuOps, ShardedDecode, ShardPlan, shard_layer, shard_rows
    from oracle.decode_ref import DecodeRef

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    bad = 0
    try:
        shape = StackShape(layers=2, hidden=512, heads=4, kv_heads=2, ffn=768, vocab=512)
        rng = np.random.default_rng(5)
        layers = [random_layer(shape, rng) for _ in range(shape.layers)]
        embed = random_rows(Q4_K, shape.vocab, shape.hidden, rng, std=1.0)
        head = random_rows(Q6_K, shape.vocab, shape.hidden, rng)
        out_norm = (1 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
        plan = ShardPlan(shape, world, rank)
        tokens = [[3, 17, 5, 100, 7, 8], [9, 0, 511, 42, 42, 1], [1, 2, 3, 4, 5, 6]]
        for collective, batch, fuse in (("nccl", 1, False), ("nccl", 3, False), ("peer", 1, False), ("peer", 3, False),
                                        ("nccl", 1, True), ("peer", 1, True)):
            ops = GpuOps(local, world=world, collective=collective, rank=rank)
            model = ShardedDecode(plan, 32, batch, [shard_layer(l, plan) for l in layers], embed,
                                  shard_rows(head, plan, "head"), out_norm, ops, fuse_norm=fuse)
            refs = [DecodeRef(shape, layers, embed, head, out_norm, 32) for _ in range(batch)]
            for pos in range(len(tokens[0])):
                model.tokens.copy_(torch.tensor([tokens[b][pos] for b in range(batch)], dtype=torch.int32))
                model.step(pos)
                got = model.logits.cpu().numpy().reshape(batch, shape.vocab)
                for b in range(batch):
                    want = refs[b].step(tokens[b][pos], pos)
                    err = np.max(np.abs(got[b] - want)) / np.max(np.abs(want))
                    if not err <= 2e-3:
                        print(f"rank {rank} {collective} batch {batch} fuse {fuse} seq {b} pos {pos}: rel err {err:.3e}",
                              flush=True)
                        bad += 1
            ops.close()
            del model
            dist.barrier()
    finally:
        dist.destroy_process_group()
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
