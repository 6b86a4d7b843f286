"""Multi-GPU host logic on CPU: shard plans, and the KV-range exchange over
gloo with world_size 2, using the oracle for each rank's partial (no GPU)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def test_sequence_plan_balances_rows(pkg):
    plan = pkg.shard.plan_sequence_shards
    lens = [int(x) for x in pkg.seeded.uniform_int(3, 4, 64, 256, 8192)]
    for world in (1, 2, 4, 8):
        shards = plan(lens, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(64))
        loads = [sum(lens[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(lens)
        assert shards == plan(lens, world)  # deterministic


def test_kv_range_plan_covers_contiguously(pkg):
    plan = pkg.shard.plan_kv_ranges
    for total, world in [(32768, 8), (100, 3), (5, 4), (0, 2), (4096, 1)]:
        r = plan(total, world)
        assert len(r) == world
        pos = 0
        for b, n in r:
            assert b == pos and n >= 0
            pos += n
        assert pos == total
        assert all(n % 32 == 0 for b, n in r if b + n < total)  # only the range at the end is ragged


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _kv_range_worker(rank, world, port, result_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    import __graft_entry__
    g = __graft_entry__.load_package()
    orc = __graft_entry__.load_oracle()
    total, pos = 1000, 999
    qkv, kc, vc = g.seeded.decode_inputs(2024, total)
    q = qkv[:1536].copy()
    b, n = g.shard.plan_kv_ranges(total, world)[rank]
    # this rank's partial over its rows (the oracle stands in for the GPU)
    m, l, o = orc.attention_partial(q, kc, vc, b, b + n)
    packed = torch.from_numpy(np.concatenate([m, l, o]).astype(np.float32))
    gathered = g.shard.all_gather_partials(packed).numpy()
    w = g.shard.packed_width(12)
    assert gathered.shape == (world, w)
    gm = gathered[:, :12]
    gl = gathered[:, 12:24]
    go = gathered[:, 24:].reshape(world, 12, 128)
    out = orc.lse_combine(gm, gl, go).reshape(-1)
    full = orc.attention(q, kc, vc, pos + 1)
    err = float(np.abs(out - full).max() / np.sqrt(np.mean(full.astype(np.float64) ** 2)))
    result_q.put((rank, err))
    dist.destroy_process_group()


def test_kv_range_exchange_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_kv_range_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res[0] < 1e-5 and res[1] < 1e-5


def _seq_shard_worker(rank, world, port, result_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    import __graft_entry__
    g = __graft_entry__.load_package()
    orc = __graft_entry__.load_oracle()
    lens = [int(x) for x in g.seeded.uniform_int(7, 4, 6, 16, 300)]
    mine = g.shard.plan_sequence_shards(lens, world)[rank]
    outs = torch.zeros((len(lens), 1536))
    for s in mine:
        qkv, kc, vc = g.seeded.decode_inputs(100 + s, 320)
        q = qkv.copy()
        orc.layer_attention(q, kc, vc, lens[s] - 1, lens[s])
        outs[s] = torch.from_numpy(q[:1536])
    dist.all_reduce(outs)  # each sequence is owned by exactly one rank
    result_q.put((rank, outs.numpy()))
    dist.destroy_process_group()


def test_sequence_sharding_gloo_world2(pkg, orc):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_seq_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    lens = [int(x) for x in pkg.seeded.uniform_int(7, 4, 6, 16, 300)]
    for s, L in enumerate(lens):
        qkv, kc, vc = pkg.seeded.decode_inputs(100 + s, 320)
        ref = qkv.copy()
        orc.layer_attention(ref, kc, vc, L - 1, L)
        assert np.array_equal(res[0][s], ref[:1536]) and np.array_equal(res[1][s], ref[:1536])


def _dropout_worker(rank, world, port, result_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    import __graft_entry__
    g = __graft_entry__.load_package()
    def report(msg):
        result_q.put((rank, msg))
        result_q.close()
        result_q.join_thread()  # flush before the hard exit below

    if rank == 1:
        # This rank leaves between steps: it never joins the exchange.
        report("left")
        os._exit(0)
    try:
        g.shard.all_gather_partials(torch.zeros(g.shard.packed_width(12)))
        report("no error")
    except Exception as e:  # the survivor learns of it through the collective's error
        report("error: " + type(e).__name__)
    os._exit(0)


def test_departed_rank_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(60)
    assert res[1] == "left"
    assert res[0].startswith("error"), res[0]
