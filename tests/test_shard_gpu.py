"""KV-range sharding of one long sequence, on the GPU.

First on one GPU with the shards emulated (each shard's rows copied to its own
cache, partials combined with gqa_lse_combine_packed), then across 2 GPUs
with NCCL (skipped when fewer GPUs are visible)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
TOL = 1e-4


def nerr(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(np.asarray(got, dtype=np.float64) - ref).max() /
                 max(np.sqrt(np.mean(ref ** 2)), 1e-30))


@pytest.mark.parametrize("world,t_max,pos", [(1, 4096, 4095), (2, 4096, 4095), (3, 1000, 700),
                                             (8, 32768, 32767), (8, 32768, 5000)])
def test_emulated_kv_shards_match_oracle(pkg, orc, cuda, world, t_max, pos):
    torch = cuda
    qkv, kc, vc = pkg.seeded.decode_inputs(900 + world + pos, t_max)
    rq, rk, rv = qkv.copy(), kc.copy(), vc.copy()
    orc.layer_attention(rq, rk, rv, pos, pos + 1)
    ranges = pkg.shard.plan_kv_ranges(t_max, world)
    width = pkg.shard.packed_width(12)
    packed = torch.empty((world, width), device="cuda")
    d_qkv = torch.from_numpy(qkv).cuda()
    locs = []
    with pkg.Context(t_max=max(n for _, n in ranges)) as ctx:
        for r, (b, n) in enumerate(ranges):
            k = torch.from_numpy(np.ascontiguousarray(kc[:, b:b + n])).cuda()
            v = torch.from_numpy(np.ascontiguousarray(vc[:, b:b + n])).cuda()
            locs.append((k, v))
            base = packed[r].data_ptr()
            ctx.decode_kv_shard(pkg.kv_of(k, v), d_qkv, pos, b, n, base, base + 48, base + 96)
        out = torch.empty(1536, device="cuda")
        ctx.lse_combine_packed(world, 12, packed, width, out)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
    assert nerr(out.cpu().numpy(), rq[:1536]) <= TOL
    for r, (b, n) in enumerate(ranges):
        k, v = locs[r]
        if b <= pos < b + n:  # the owner appended the new row
            assert np.abs(k[:, pos - b].cpu().numpy() - rk[:, pos]).max() <= 1e-5
            assert np.array_equal(v[:, pos - b].cpu().numpy(), rv[:, pos])
        else:  # other shards are untouched
            assert np.array_equal(k.cpu().numpy(), kc[:, b:b + n])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _nccl_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    import __graft_entry__
    g = __graft_entry__.load_package()
    t_max, pos = 8192, 8191
    qkv, kc, vc = g.seeded.decode_inputs(77, t_max)
    b, n = g.shard.plan_kv_ranges(t_max, world)[rank]
    with g.Context(t_max=n, device=rank) as ctx:
        k = torch.from_numpy(np.ascontiguousarray(kc[:, b:b + n])).cuda()
        v = torch.from_numpy(np.ascontiguousarray(vc[:, b:b + n])).cuda()
        dec = g.shard.KvShardDecoder(ctx, k, v, b, n)
        out = torch.empty(1536, device="cuda")
        dec.step(torch.from_numpy(qkv).cuda(), pos, out)
        torch.cuda.synchronize()
        q.put((rank, out.cpu().numpy()))
    dist.barrier()
    dist.destroy_process_group()


def test_kv_shards_over_two_gpus_nccl(pkg, orc, cuda):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    qkv, kc, vc = pkg.seeded.decode_inputs(77, 8192)
    rq = qkv.copy()
    orc.layer_attention(rq, kc, vc, 8191, 8192)
    for r in range(2):
        assert nerr(res[r], rq[:1536]) <= TOL
