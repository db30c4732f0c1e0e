"""Host-side multi-GPU logic on CPU: request assignment, result gather and the split-KV
exchange, with world_size-2 gloo process groups (127.0.0.1)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import inputs as gin
import oracle
from mdflash_b200 import sharding as S


def test_request_specs_match_config():
    specs = S.request_specs(64, seed=0)
    assert len(specs) == 64
    assert all(1024 <= s.prefix <= 32768 for s in specs)
    assert {s.budget for s in specs} <= {64, 128, 256, 512}
    assert len({s.seed for s in specs}) == 64
    assert S.request_specs(64, seed=0) == specs


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_lpt_assignment_partitions_and_balances(world):
    specs = S.request_specs(64, seed=1)
    costs = [S.request_cost(s) for s in specs]
    parts = S.assign_requests(costs, world)
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(64))
    loads = [sum(costs[i] for i in p) for p in parts]
    # LPT bound: max load <= mean + largest job
    assert max(loads) <= sum(costs) / world + max(costs) + 1e-6
    assert S.assign_requests(costs, world) == parts


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_gemm_chunk_of_each_rank(world):
    """The batched verify forward's projection chunk for each rank's tree rows: at most 2048
    rows, a multiple of 128, the fewest chunks, and under 128 padding rows per chunk."""
    from mdflash_b200.runner import gemm_chunk
    specs = S.request_specs(64, seed=0)
    parts = S.assign_requests([S.request_cost(s) for s in specs], world)
    for part in parts:
        rows = sum(specs[i].budget + 1 for i in part)
        c = gemm_chunk(rows)
        pieces = -(-rows // c)
        assert c <= 2048 and c % 128 == 0
        assert pieces == -(-rows // 2048)
        assert pieces * c - rows < 128 * pieces
    if world == 1:
        assert sum(s.budget + 1 for s in specs) == 18112 and gemm_chunk(18112) == 2048
    assert gemm_chunk(1) == 128 and gemm_chunk(2049) == 1152
    with pytest.raises(ValueError):
        gemm_chunk(0)


def test_result_records_roundtrip():
    rec = S.pack_result(7, 257, [0, 3, 9], 1234, time_ns=55, rank=1)
    d = S.unpack_result(rec)
    assert d == dict(index=7, rank=1, n_nodes=257, n_accepted=3, next_token=1234, time_ns=55,
                     accepted=[0, 3, 9])


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("prefix,n", [(131072, 513), (4096, 65), (1000, 33)])
def test_shard_ranges_cover_keys_once(world, prefix, n):
    if prefix < world * 128:
        pytest.skip("prefix shorter than one aligned shard per rank")
    ranges = [S.shard_range(prefix, n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == prefix + n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    assert all(e > b for b, e in ranges)
    assert all(b % 128 == 0 for b, _ in ranges)
    assert S.owner_rank(world) == world - 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial_reference(q, k, v, vis, past, kb, ke):
    """fp32 partial (O unnormalised, m in log2 units of scaled scores, l) over keys [kb, ke):
    the quantities ddt_tree_attn_partial produces (test-only CPU restatement)."""
    hq, n, d = q.shape
    g = hq // k.shape[0]
    kk = k.repeat_interleave(g, 0)[:, kb:ke].float()
    vv = v.repeat_interleave(g, 0)[:, kb:ke].float()
    s = torch.einsum("hnd,hsd->hns", q.float(), kk) * (d ** -0.5) * 1.4426950408889634
    keys = torch.arange(kb, ke)
    allowed = torch.ones((n, ke - kb), dtype=torch.bool)
    tree = keys >= past
    if tree.any():
        allowed[:, tree] = torch.from_numpy(vis)[:, keys[tree] - past]
    s = s.masked_fill(~allowed[None], float("-inf"))
    m = s.amax(-1)
    p = torch.exp2(s - m[..., None].clamp_min(-1e30))
    p = torch.nan_to_num(p)
    lsum = p.sum(-1)
    o = torch.einsum("hns,hsd->hnd", p, vv)
    # [N, Hq] row order like the kernel's partials
    return o.transpose(0, 1).reshape(n * hq, d), m.transpose(0, 1).reshape(-1), lsum.transpose(0, 1).reshape(-1)


def _merge_reference(o, m, l):
    M = m.amax(0)
    w = torch.where(m == float("-inf"), torch.zeros_like(m), torch.exp2(m - M))
    return (o * w[..., None]).sum(0) / (l * w).sum(0)[..., None]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # result gather: rank r holds requests r, r + world, ...
        recs = torch.stack([S.pack_result(i, 33 + i, [0, i % 5 + 1], 100 + i, rank=rank)
                            for i in range(rank, 10, world)])
        allr = S.gather_results(recs)
        got = [S.unpack_result(r) for r in allr]
        assert [g["index"] for g in got] == list(range(10))
        assert all(g["rank"] == g["index"] % world for g in got)
        # split-KV exchange over a sharded prefix
        spec = gin.ATTN_CASES[1]
        qq, kk, vv, parents = gin.attn_inputs(spec)
        vis = oracle.visibility(parents)
        past, n = spec["past"], spec["n"]
        kb, ke = S.shard_range(past, n, world, rank, align=64)
        o, m, l = _partial_reference(qq, kk, vv, vis, past, kb, ke)
        og, mg, lg = S.exchange_partials(o, m, l)
        merged = _merge_reference(og, mg, lg).view(n, qq.shape[0], -1)
        full = oracle.tree_attention(qq, kk, vv, vis, past)
        err = ((merged - full).abs().max() / full.abs().max()).item()
        # the same partials, one per row, through the no-copy gather
        og2, mg2, lg2 = S.gather_partials(o, m, l)
        assert og2.shape == (world,) + tuple(o.shape) and mg2.shape == (world, m.shape[0])
        merged2 = _merge_reference(og2, mg2, lg2).view(n, qq.shape[0], -1)
        err = max(err, ((merged2 - full).abs().max() / full.abs().max()).item())
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


def test_gather_and_splitkv_exchange_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(world))
    assert max(errs.values()) < 1e-5, errs
