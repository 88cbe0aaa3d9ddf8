"""Split-KV decode over NCCL through the C ABI alone (g4a_dist_init, g4a_decode_attn_splitkv,
g4a_dist_allgather_host) against the fp64 oracle.

One GPU: a one-rank communicator (the whole cache is the rank's slice).  Two GPUs (skipped
otherwise): two processes, one per GPU, with no torch.distributed -- the NCCL unique id travels
over a multiprocessing queue -- split a 20k-token sequence, run several steps, and bootstrap the
peer-memory exchange (g4a_splitkv_exchange_merge) with g4a_dist_allgather_host.  A rank that
stays out of a step (alive, with nothing in flight) makes the other rank's g4a_sync end with
G4A_ETIMEOUT and abort its communicator; that rank's context stays usable.  NVLS is off
(NCCL_NVLS_ENABLE=0) in these processes."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import g4attn
from g4attn import G4AError, dist as gdist
from gpu_helpers import assert_attention_close, dev, host

pytestmark = pytest.mark.gpu


def _sequence(L, seed=5):
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((L, 1, 256)).astype(np.float32).astype(np.float16)
    v = rng.standard_normal((L, 1, 256)).astype(np.float32).astype(np.float16)
    return k, v


def _query(step, seed=19):
    rng = np.random.default_rng(seed + step)
    q = rng.standard_normal((8, 256)).astype(np.float32)
    return q / np.sqrt((q * q).mean(-1, keepdims=True))


def test_one_rank_communicator(oracle):
    L = 5000
    k, v = _sequence(L)
    with g4attn.Context(0) as c:
        c.dist_init(0, 1, g4attn.dist_unique_id(), 60000)
        assert c.dist_info() == (0, 1)
        dec = gdist.CabiSplitKVDecoder(c)
        kd, vd = dev(k.view(np.uint16)).view(torch.float16), dev(v.view(np.uint16)).view(torch.float16)
        for step in range(1, 3):
            out = torch.full((8, 256), float("nan"), device="cuda")
            dec.step(dev(_query(step)), kd, vd, out, begin=0, end=L, kv_len_total=L)
            c.sync()
            ref = oracle.decode_attn_f64(_query(step), k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=L)
            assert_attention_close(host(out), ref, what=f"one-rank step {step}")
        assert c.dist_allgather_host(b"abc") == [b"abc"]
        c.dist_destroy()
        assert c.dist_info() == (-1, 0)
        with pytest.raises(G4AError):
            dec.step(dev(_query(1)), kd, vd, out, begin=0, end=L, kv_len_total=L)


def _worker(rank, world, L, steps, id_q, out_q, skip_last, release):
    import sys
    from pathlib import Path

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root / "gemma4-webgpu_b200"), str(root), str(root / "tests")]
    import numpy as np
    import torch

    import g4attn
    from g4attn import G4AError, dist as gd

    torch.cuda.set_device(rank)
    ctx = None
    try:
        if rank == 0:
            uid = g4attn.dist_unique_id()
            for _ in range(world - 1):
                id_q.put(uid)
        else:
            uid = id_q.get(timeout=60)
        ctx = g4attn.Context(rank)
        ctx.dist_init(rank, world, uid, 60000)
        k, v = _sequence(L)
        b, e = gd.splitkv_ranges(L, world, 64)[rank]
        kd = torch.from_numpy(k[b:e].view(np.uint16)).cuda().view(torch.float16)
        vd = torch.from_numpy(v[b:e].view(np.uint16)).cuda().view(torch.float16)
        dec = gd.CabiSplitKVDecoder(ctx, timeout_ms=20000)
        outs = []
        for step in range(1, steps + 1):
            q = torch.from_numpy(_query(step)).cuda()
            out = torch.zeros((8, 256), device="cuda")
            dec.step(q, kd, vd, out, begin=b, end=e, kv_len_total=L)
            ctx.sync(20000)
            outs.append(out.cpu().numpy())
        # the peer-memory exchange, bootstrapped over the same communicator
        peer = gd.CabiPeerSplitKVDecoder(ctx, timeout_ms=20000)
        q = torch.from_numpy(_query(steps + 1)).cuda()
        out = torch.zeros((8, 256), device="cuda")
        peer.step(q, kd, vd, out, begin=b, end=e, kv_len_total=L)
        ctx.sync(20000)
        outs.append(out.cpu().numpy())
        peer.close()
        timed_out = None
        if skip_last:
            # rank 1 stays out of this step (alive, nothing in flight); rank 0's collective cannot
            # complete, its sync deadline aborts the communicator, its context stays usable
            if rank == 0:
                q = torch.from_numpy(_query(99)).cuda()
                out = torch.zeros((8, 256), device="cuda")
                try:
                    dec.step(q, kd, vd, out, begin=b, end=e, kv_len_total=L)
                    ctx.sync(3000)
                    timed_out = "no error"
                except G4AError as ex:
                    timed_out = ex.status_name + ": " + str(ex)
                single = torch.zeros((8, 256), device="cuda")
                ctx.decode_attn(q, kd, vd, single, num_q_heads=8, num_kv_heads=1, head_dim=256, seq_len=e - b)
                ctx.sync(20000)
                release.set()
            else:
                release.wait(120)
        out_q.put((rank, outs, timed_out, None))
    except Exception as ex:  # reported to the parent
        out_q.put((rank, None, None, repr(ex)))
        release.set()
    finally:
        if ctx is not None:
            ctx.close()


def _run(world, L, steps, skip_last):
    ctxm = mp.get_context("spawn")
    id_q, out_q, release = ctxm.Queue(), ctxm.Queue(), ctxm.Event()
    procs = [ctxm.Process(target=_worker, args=(r, world, L, steps, id_q, out_q, skip_last, release))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [out_q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return sorted(results)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.timeout(300)
def test_two_gpu_cabi_splitkv_matches_oracle(oracle):
    L, steps = 20000, 3
    k, v = _sequence(L)
    for rank, outs, _, err in _run(2, L, steps, False):
        assert err is None, (rank, err)
        for step, o in enumerate(outs, start=1):
            ref = oracle.decode_attn_f64(_query(step), k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=L)
            assert_attention_close(o, ref, what=f"rank {rank} step {step}")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.timeout(300)
def test_two_gpu_missing_rank_times_out_and_aborts():
    res = _run(2, 20000, 1, True)
    for rank, outs, timed_out, err in res:
        assert err is None, (rank, err)
    assert res[0][2] is not None and res[0][2].startswith("G4A_ETIMEOUT"), res[0][2]
    assert "aborted" in res[0][2]
