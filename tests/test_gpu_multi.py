"""Split-KV (sequence-sharded prefix) attention on GPUs: partials of every shard, the
exchange and ddt_attn_merge must reproduce the single-GPU tree attention.  With one GPU the
shards run in one process (the exchange is a stack, or the peer exchange of a single rank);
with two or more GPUs the shards run in NCCL processes, one per GPU, and the exchange over
NVLink peer memory (PeerExchange) must give exactly the NCCL all-gather's output."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import inputs as gin
import oracle
from mdflash_b200 import kernels as K
from mdflash_b200 import sharding as S

pytestmark = pytest.mark.gpu
P, N = 4096, 129


def _data(device):
    g = torch.Generator().manual_seed(0)
    sc = 128 ** -0.5
    q = (torch.randn((N, 32, 128), generator=g) * sc).to(torch.bfloat16).to(device)
    k = (torch.randn((8, P + N, 128), generator=g) * sc).to(torch.bfloat16).to(device)
    v = torch.randn((8, P + N, 128), generator=g).to(torch.bfloat16).to(device)
    parents = gin.random_tree(N, 3)
    bits = torch.from_numpy(oracle.ancestor_bits(parents).view(np.int32)).to(device)
    return q, k, v, bits


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()


@pytest.mark.parametrize("world", [1, 2, 4])
def test_splitkv_shards_in_one_process(cuda_device, world):
    q, k, v, bits = _data(cuda_device)
    full = K.tree_attention(q, k, v, bits, P)
    parts = []
    for r in range(world):
        kb, ke = S.shard_range(P, N, world, r)
        parts.append(K.tree_attention_partial(q, k[:, kb:ke].contiguous(), v[:, kb:ke].contiguous(),
                                              kb, ke, bits, P))
    # each shard yields [S, rows, ...] partials (S in-GPU key splits)
    merged = K.attn_merge(torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts]),
                          torch.cat([p[2] for p in parts]), N, 32)
    torch.cuda.synchronize()
    assert _rel(merged, full) <= 1e-2
    assert _rel(S.splitkv_attention(q, k, v, 0, P + N, bits, P), full) <= 1e-2


@pytest.mark.parametrize("world", [1, 2, 3])
def test_merged_partials_per_shard(cuda_device, world):
    """One in-GPU-merged partial per row and shard (balanced work items inside each shard),
    then the cross-shard merge."""
    q, k, v, bits = _data(cuda_device)
    full = K.tree_attention(q, k, v, bits, P)
    parts = [K.tree_attention_partial_merged(q, k[:, kb:ke].contiguous(), v[:, kb:ke].contiguous(),
                                             kb, ke, bits, P)
             for kb, ke in (S.shard_range(P, N, world, r) for r in range(world))]
    merged = K.attn_merge(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]),
                          torch.stack([p[2] for p in parts]), N, 32)
    torch.cuda.synchronize()
    assert _rel(merged, full) <= 1e-2


def test_peer_exchange_one_rank(cuda_device):
    """PeerExchange without a process group (world 1): the push into its own buffer and the
    counter-waiting merge give exactly ddt_attn_merge's output, call after call (the two
    buffer parities alternate)."""
    q, k, v, bits = _data(cuda_device)
    full = K.tree_attention(q, k, v, bits, P)
    x = S.PeerExchange(N, 32, cuda_device)
    try:
        for _ in range(3):
            o, m, l = K.tree_attention_partial_merged(q, k, v, 0, P + N, bits, P)
            ref = K.attn_merge(o[None], m[None], l[None], N, 32)
            got = x.exchange_merge(o, m, l)
            torch.cuda.synchronize()
            assert torch.equal(got, ref)
            assert _rel(got, full) <= 1e-2
            assert int(x.status.item()) == 0
            again = x.attend(q, k, v, 0, P + N, bits, P)
            torch.cuda.synchronize()
            assert torch.equal(again, ref)
    finally:
        x.close()


@pytest.mark.parametrize("past", [4096, 20000])
def test_peer_exchange_fused_merge_one_rank(cuda_device, past):
    """PeerExchange.attend (world 1): the shard attention's own merge stores into the receive
    buffer.  At 20000 keys the K / V exceed L2 and the shard runs the uniform-split plan,
    whose merge kernel pushes; at 4096 the balanced plan merges locally and a copy kernel
    pushes.  Both equal partial_merged + ddt_attn_merge exactly, call after call."""
    g = torch.Generator().manual_seed(1)
    sc = 128 ** -0.5
    q = (torch.randn((N, 32, 128), generator=g) * sc).to(torch.bfloat16).to(cuda_device)
    k = (torch.randn((8, past + N, 128), generator=g) * sc).to(torch.bfloat16).to(cuda_device)
    v = torch.randn((8, past + N, 128), generator=g).to(torch.bfloat16).to(cuda_device)
    bits = torch.from_numpy(oracle.ancestor_bits(gin.random_tree(N, 4)).view(np.int32)).to(
        cuda_device)
    o, m, l = K.tree_attention_partial_merged(q, k, v, 0, past + N, bits, past)
    ref = K.attn_merge(o[None], m[None], l[None], N, 32)
    full = K.tree_attention(q, k, v, bits, past)
    x = S.PeerExchange(N, 32, cuda_device)
    try:
        for _ in range(3):
            got = S.splitkv_attention(q, k, v, 0, past + N, bits, past, exchange=x)
            torch.cuda.synchronize()
            assert torch.equal(got, ref)
            assert int(x.status.item()) == 0
        assert _rel(got, full) <= 1e-2
    finally:
        x.close()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        q, k, v, bits = _data(dev)
        kb, ke = S.shard_range(P, N, world, rank)
        ks, vs = k[:, kb:ke].contiguous(), v[:, kb:ke].contiguous()
        out = S.splitkv_attention(q, ks, vs, kb, ke, bits, P)
        full = K.tree_attention(q, k, v, bits, P)
        # the same exchange over NVLink peer memory: identical output, several calls in a row
        x = S.PeerExchange(N, 32, dev)
        same = True
        try:
            for _ in range(3):
                peer = S.splitkv_attention(q, ks, vs, kb, ke, bits, P, exchange=x)
                torch.cuda.synchronize()
                same = same and torch.equal(peer, out) and int(x.status.item()) == 0
        finally:
            x.close()
        torch.cuda.synchronize()
        q_out.put((rank, _rel(out, full) if same else 1.0))
    finally:
        dist.destroy_process_group()


def test_splitkv_over_nccl():
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    ctx = mp.get_context("spawn")
    qo = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, qo)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(qo.get(timeout=5) for _ in range(world))
    assert max(errs.values()) <= 1e-2, errs
