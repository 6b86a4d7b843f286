"""KV-range sharding of one long sequence, on the GPU.

First on one GPU with the shards emulated (each shard's rows copied to its own
cache, partials combined with gqa_lse_combine_packed), then across 2 GPUs
with NCCL, and the peer-memory exchange (gqa_decode_kv_shard_exchange): on
one GPU as a group of one (several steps, both inbox parities), its bounded
wait when a peer never arrives, and across 2 GPUs (skipped when fewer GPUs
are visible)."""
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


def _oracle_steps(pkg, orc, seed, t_max, positions):
    """Oracle outputs for consecutive decode steps of one sequence, each step
    appending its row (the same qkv row at each position)."""
    qkv, kc, vc = pkg.seeded.decode_inputs(seed, t_max)
    rk, rv, outs = kc.copy(), vc.copy(), []
    for pos in positions:
        rq = qkv.copy()
        orc.layer_attention(rq, rk, rv, pos, pos + 1)
        outs.append(rq[:1536].copy())
    return qkv, kc, vc, outs


def test_exchange_group_of_one_steps(pkg, orc, cuda):
    torch = cuda
    t_max, positions = 8192, [6000, 6001, 6002, 6003]
    qkv, kc, vc, ref = _oracle_steps(pkg, orc, 31, t_max, positions)
    with pkg.Context(t_max=t_max) as ctx:
        k = torch.from_numpy(kc).cuda()
        v = torch.from_numpy(vc).cuda()
        dec = pkg.shard.KvShardExchangeDecoder(ctx, k, v, 0, t_max)
        d_qkv = torch.from_numpy(qkv).cuda()
        out = torch.empty(1536, device="cuda")
        for pos, r in zip(positions, ref):
            dec.step(d_qkv, pos, out)
            torch.cuda.synchronize()
            assert ctx.device_status() == 0
            assert nerr(out.cpu().numpy(), r) <= TOL
        dec.close()


def test_exchange_absent_peer_times_out(pkg, cuda):
    """A group of two whose second rank never runs: the kernel's wait for its
    flag gives up after its budget (~1 s), raises the wait-timeout status bit
    and leaves the output unwritten; the GPU stays usable."""
    torch = cuda
    t_max = 1024
    qkv, kc, vc = pkg.seeded.decode_inputs(5, t_max)
    with pkg.Context(t_max=t_max) as ctx:
        x = pkg.gqa.Exchange(ctx, 0, 2)
        x.open([x.handle, x.handle])  # the absent rank's inbox maps to our own
        k = torch.from_numpy(kc).cuda()
        v = torch.from_numpy(vc).cuda()
        out = torch.full((1536,), 7.0, device="cuda")
        x.step(pkg.kv_of(k, v), torch.from_numpy(qkv).cuda(), 700, 0, t_max, out)
        torch.cuda.synchronize()
        st = ctx.device_status()
        assert st & pkg.gqa.STATUS_WAIT_TIMEOUT
        assert bool((out == 7.0).all())
        x.destroy()
        # the context still works afterwards
        out2 = torch.empty(1536, device="cuda")
        ctx.layer_attention_out(pkg.kv_of(k, v), torch.from_numpy(qkv).cuda(), 700, 701, out2)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0


TWO_GPU_POSITIONS = [2000, 4095, 4096, 8191]


def _exchange_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    # gloo only swaps the inbox handles; the data path is the kernel's NVLink stores
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    import __graft_entry__
    g = __graft_entry__.load_package()
    # 2000 and 4095: rank 1's shard [4096, 8192) attends no row (it still takes
    # part); 4096: rank 1 holds the new row and attends only it; 8191: both full.
    t_max, positions = 8192, TWO_GPU_POSITIONS
    qkv, kc, vc = g.seeded.decode_inputs(78, t_max)
    b, n = g.shard.plan_kv_ranges(t_max, world)[rank]
    outs = []
    with g.Context(t_max=n, device=rank) as ctx:
        k = torch.from_numpy(np.ascontiguousarray(kc[:, b:b + n])).cuda()
        v = torch.from_numpy(np.ascontiguousarray(vc[:, b:b + n])).cuda()
        dec = g.shard.KvShardExchangeDecoder(ctx, k, v, b, n)
        d_qkv = torch.from_numpy(qkv).cuda()
        out = torch.empty(1536, device="cuda")
        for pos in positions:
            dec.step(d_qkv, pos, out)
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy().copy())
        status = ctx.device_status()
        dist.barrier()  # no rank unmaps its inbox while a peer may still write to it
        dec.close()
        q.put((rank, status, outs))
    dist.barrier()
    dist.destroy_process_group()


def test_kv_shards_over_two_gpus_exchange(pkg, orc, cuda):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (st, outs) for r, st, outs in (q.get(timeout=300) for _ in range(2))}
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    _, _, _, ref = _oracle_steps(pkg, orc, 78, 8192, TWO_GPU_POSITIONS)
    for r in range(2):
        st, outs = res[r]
        assert st == 0
        for got, want in zip(outs, ref):
            assert nerr(got, want) <= TOL


def _prefill_worker(rank, world, seqs, S, q):
    import torch
    torch.cuda.set_device(rank)
    import __graft_entry__
    g = __graft_entry__.load_package()
    mine = g.shard.plan_sequence_shards([S] * seqs, world)[rank]
    res = {}
    with g.Context(t_max=S, device=rank) as ctx:
        for s in mine:
            x = g.seeded.normal(4400 + s, g.seeded.PREFILL_Q, S * 2048).reshape(1, S, 2048)
            d_x = torch.from_numpy(x).cuda()
            out = torch.zeros((1, S, 1536), device="cuda")
            kc = torch.zeros((1, 2, S, 128), device="cuda")
            vc = torch.zeros((1, 2, S, 128), device="cuda")
            kp = torch.tensor([kc.data_ptr()], dtype=torch.int64, device="cuda")
            vp = torch.tensor([vc.data_ptr()], dtype=torch.int64, device="cuda")
            ctx.prefill_bf16(1, S, d_x, out, kp, vp)
            torch.cuda.synchronize()
            res[s] = (out.cpu().numpy()[0], kc.cpu().numpy()[0], vc.cpu().numpy()[0])
        status = ctx.device_status()
    q.put((rank, status, res))


def test_prefill_sequences_over_two_gpus(pkg, orc, cuda):
    """Causal prefill sharded by sequence: four prompts dealt to two GPUs
    (no collective on the data path), each GPU's outputs and appended cache
    rows checked against the oracle on the same bf16 operands."""
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import test_prefill_gpu as tp
    seqs, S = 4, 256
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_prefill_worker, args=(r, 2, seqs, S, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        rank, st, res = q.get(timeout=300)
        assert st == 0, rank
        assert len(res) == seqs // 2, rank  # equal prompts: two per GPU
        got.update(res)
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert sorted(got) == list(range(seqs))
    for s in range(seqs):
        x = pkg.seeded.normal(4400 + s, pkg.seeded.PREFILL_Q, S * 2048).reshape(S, 2048)
        out, kc, vc = got[s]
        tp.check_sequence(torch, orc, x, out, list(range(0, S, 3)) + [S - 1], kc, vc)
