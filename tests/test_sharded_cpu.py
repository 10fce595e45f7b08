"""Row-sharded decode orchestration on CPU ranks (gloo), world size 2.

ShardedDecode with the float64 NumpyOps arithmetic runs as two spawned gloo
ranks (127.0.0.1); each rank owns half of every linear's rows, half of the
heads and half of the LM head. Its gathered logits must equal the unsharded
restatement (oracle/decode_ref.py) for every position, for one sequence and
for a batch of three (which exercises the [rank][batch][rows] gather
re-layout) -- both on activation codes and in the batched fp32 mode whose
linears take the tile path on the device --, to 1e-9 relative. Also checks the plan's row ranges and its
refusal of shapes that do not divide.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from cybel_b200.decode import StackShape

TINY = StackShape(layers=2, hidden=512, heads=4, kv_heads=2, ffn=768, vocab=512)
TOKENS = [[3, 17, 5, 100, 7], [9, 0, 511, 42, 42], [1, 2, 3, 4, 5]]


def _weights():
    from cybel_b200.decode import random_layer, random_rows
    from cybel_b200.formats import Q4_K, Q6_K

    rng = np.random.default_rng(11)
    layers = [random_layer(TINY, rng) for _ in range(TINY.layers)]
    embed = random_rows(Q4_K, TINY.vocab, TINY.hidden, rng, std=1.0)
    head = random_rows(Q6_K, TINY.vocab, TINY.hidden, rng)
    out_norm = (1 + 0.1 * rng.standard_normal(TINY.hidden)).astype(np.float32)
    return layers, embed, head, out_norm


def _worker(rank, world, port, batch, q, fuse=False, tile=False):
    import torch.distributed as dist

    from cybel_b200.sharded import ShardedDecode, ShardPlan, shard_layer, shard_rows
    from sharded_cpu_ops import NumpyOps

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layers, embed, head, out_norm = _weights()
        plan = ShardPlan(TINY, world, rank)
        model = ShardedDecode(plan, 16, batch, [shard_layer(l, plan) for l in layers], embed,
                              shard_rows(head, plan, "head"), out_norm, NumpyOps(world), fuse_norm=fuse, tile=tile)
        assert model.tile == tile
        outs = []
        for pos in range(len(TOKENS[0])):
            model.tokens[:] = [TOKENS[b][pos] for b in range(batch)]
            model.step(pos)
            outs.append(model.logits.copy())
        q.put((rank, np.stack(outs)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("batch,fuse,tile", [(1, False, False), (3, False, False), (1, True, False), (3, False, True)])
def test_two_rank_sharded_decode_equals_unsharded(batch, fuse, tile):
    import multiprocessing as mp

    from oracle.decode_ref import DecodeRef

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, q, fuse, tile)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    layers, embed, head, out_norm = _weights()
    for b in range(batch):
        ref = DecodeRef(TINY, layers, embed, head, out_norm, 16)
        for pos in range(len(TOKENS[0])):
            want = ref.step(TOKENS[b][pos], pos)
            for r in range(2):
                row = got[r][pos][b * TINY.vocab:(b + 1) * TINY.vocab]
                assert np.max(np.abs(row - want)) <= 1e-9 * np.max(np.abs(want)), (r, b, pos)


def test_shard_plan_rows_and_refusals():
    from cybel_b200.decode import LLAMA3_70B
    from cybel_b200.sharded import ShardPlan

    p = ShardPlan(LLAMA3_70B, 8, 3)
    assert p.heads == 8 and p.kv_heads == 1
    assert p.row_range("wq") == (3 * 1024, 4 * 1024)
    assert p.row_range("wk") == (3 * 128, 4 * 128)
    assert p.row_range("w_gate") == (3 * 3584, 4 * 3584)
    assert p.row_range("w_down") == (3 * 1024, 4 * 1024)
    assert p.row_range("head") == (3 * 16032, 4 * 16032)
    with pytest.raises(ValueError):
        ShardPlan(LLAMA3_70B, 16, 0)  # 8 kv heads do not split 16 ways
    with pytest.raises(ValueError):
        ShardPlan(TINY, 3, 0)
