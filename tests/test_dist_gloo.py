"""Multi-rank host logic on CPU with gloo (world size 2): the split-KV exchange (partials in the
library's m | l | o layout, all-gathered in rank order, merged) and the batched sharding
(every sequence on exactly one rank, same assignment computed on every rank)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, out_q):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root / "gemma4-webgpu_b200"), str(root)]
    import torch
    import torch.distributed as dist

    from g4attn.dist import decode_cost_bytes, lpt_shard, merge_partials_host, partial_floats, splitkv_ranges
    from g4attn import synth
    from oracle import oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        qv, k, v, L = q
        b, e = splitkv_ranges(L, world)[rank]
        m, l_, o = orc.decode_partial_f64(qv, k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_begin=b,
                                          kv_end=e, kv_len=L)
        part = np.concatenate([m / np.log(2.0), l_, o.reshape(-1)]).astype(np.float32)
        mine = torch.from_numpy(part)
        gathered = torch.zeros(world * partial_floats(8, 256))
        dist.all_gather_into_tensor(gathered, mine)
        merged = merge_partials_host(gathered.numpy().reshape(world, -1), 8, 256)

        lengths = synth.batched_lengths(2, 64)
        bins = lpt_shard(decode_cost_bytes(lengths), world)
        mine_ids = torch.tensor(bins[rank] + [-1] * (64 - len(bins[rank])), dtype=torch.int64)
        all_ids = [torch.zeros(64, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(all_ids, mine_ids)
        ids = sorted(int(i) for t in all_ids for i in t if i >= 0)
        out_q.put((rank, merged, ids))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_splitkv_and_sharding(oracle):
    rng = np.random.default_rng(17)
    L = 3000
    q = rng.standard_normal((8, 256)).astype(np.float32)
    q /= np.sqrt((q * q).mean(-1, keepdims=True))
    k = oracle.f32_to_f16(rng.standard_normal((L, 1, 256)).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal((L, 1, 256)).astype(np.float32))
    full = oracle.decode_attn_f64(q, k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=L)
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, (q, k, v, L), out_q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [out_q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, merged, ids in results:
        assert np.abs(merged - full).max() < 1e-5, rank
        assert ids == list(range(64)), rank
