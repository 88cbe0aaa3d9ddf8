"""Split-KV exchange over peer memory (g4a_splitkv_exchange_merge) against the fp64 oracle.

One GPU: a single-rank exchange (the kernel pushes to and waits on its own buffer), and a flag
that no rank ever sets, which must end the bounded wait with an error and a zeroed output.
Two GPUs (skipped otherwise): two processes, one per GPU, exchange their partials of a 20k-token
sequence over NVLink for several steps with a different query each step (both buffer parities)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from g4attn import G4AError, dist as gdist
from gpu_helpers import assert_attention_close, dev, host

pytestmark = pytest.mark.gpu


def _sequence(L, seed=5):
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((L, 1, 256)).astype(np.float32).astype(np.float16)
    v = rng.standard_normal((L, 1, 256)).astype(np.float32).astype(np.float16)
    return k, v


def _query(step, seed=9):
    rng = np.random.default_rng(seed + step)
    q = rng.standard_normal((8, 256)).astype(np.float32)
    return q / np.sqrt((q * q).mean(-1, keepdims=True))


def test_single_rank_exchange(ctx, oracle):
    from g4attn._lib import load

    L = 3000
    k, v = _sequence(L)
    kd, vd = dev(k.view(np.uint16)).view(torch.float16), dev(v.view(np.uint16)).view(torch.float16)
    nbytes = int(load().g4a_exchange_buffer_bytes(1, 8, 256))
    buf = ctx.alloc(nbytes)
    try:
        ctx.memset(buf, 0, nbytes)
        part = torch.empty(gdist.partial_floats(8, 256), device="cuda")
        out = torch.full((8, 256), float("nan"), device="cuda")
        for step in range(1, 4):
            q = _query(step)
            ctx.decode_attn_partial(dev(q), kd, vd, part, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_begin=0,
                                    kv_end=L, kv_len_total=L)
            ctx.splitkv_exchange_merge(part, [buf], 0, step, out, num_q_heads=8, head_dim=256)
            ctx.sync()
            ref = oracle.decode_attn_f64(q, k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=L)
            assert_attention_close(host(out), ref, what=f"single-rank exchange step {step}")
    finally:
        ctx.sync()
        ctx.free(buf)


def test_missing_peer_times_out_with_error(ctx):
    """World 2 with nobody playing rank 1: the wait for its flag ends after its bound, the output
    is zeroed and g4a_sync reports the error; the context stays usable."""
    from g4attn._lib import load

    nbytes = int(load().g4a_exchange_buffer_bytes(2, 8, 256))
    bufs = [ctx.alloc(nbytes), ctx.alloc(nbytes)]
    try:
        for b in bufs:
            ctx.memset(b, 0, nbytes)
        part = torch.zeros(gdist.partial_floats(8, 256), device="cuda")
        out = torch.full((8, 256), 7.0, device="cuda")
        ctx.splitkv_exchange_merge(part, bufs, 0, 1, out, num_q_heads=8, head_dim=256)
        with pytest.raises(G4AError) as ei:
            ctx.sync()
        assert "peer" in str(ei.value)
        assert not host(out).any()
        ctx.sync()
    finally:
        for b in bufs:
            ctx.free(b)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, L, steps, out_q):
    import datetime
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root / "gemma4-webgpu_b200"), str(root), str(root / "tests")]
    import numpy as np
    import torch
    import torch.distributed as tdist

    import g4attn
    from g4attn import dist as gd

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    tdist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        k, v = _sequence(L)
        b, e = gd.splitkv_ranges(L, world, 64)[rank]
        ctx = g4attn.Context(rank)
        kd = torch.from_numpy(k[b:e].view(np.uint16)).cuda().view(torch.float16)
        vd = torch.from_numpy(v[b:e].view(np.uint16)).cuda().view(torch.float16)
        dec = gd.PeerSplitKVDecoder(ctx)
        outs = []
        for step in range(1, steps + 1):
            q = torch.from_numpy(_query(step)).cuda()
            out = torch.zeros((8, 256), device="cuda")
            dec.step(q, kd, vd, out, begin=b, end=e, kv_len_total=L)
            ctx.sync()
            outs.append(out.cpu().numpy())
        dec.close()
        ctx.close()
        out_q.put((rank, outs, None))
    except Exception as ex:  # reported to the parent
        out_q.put((rank, None, repr(ex)))
    finally:
        tdist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.timeout(300)
def test_two_gpu_exchange_matches_oracle(oracle):
    L, steps = 20000, 4
    k, v = _sequence(L)
    ctxm = mp.get_context("spawn")
    out_q = ctxm.Queue()
    port = _free_port()
    procs = [ctxm.Process(target=_worker, args=(r, 2, port, L, steps, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [out_q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, outs, err in results:
        assert err is None, (rank, err)
        for step, o in enumerate(outs, start=1):
            ref = oracle.decode_attn_f64(_query(step), k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=L)
            assert_attention_close(o, ref, what=f"rank {rank} step {step}")
