"""Multi-GPU partitioning of the DDTree verify path (one process per GPU).

Two modes, both without any data-path collective inside the verify step except the one
split-KV exchange:

* Request data parallelism.  The reference shards its dataset rank-strided
  (benchmark.py:436, ``indices = range(rank, len, world)``) and gathers pickled per-request
  results to rank 0 with ``gather_object`` (distributed.py:55-64).  Here requests are
  assigned by longest-processing-time first on a cost model of the verify step (attention
  grows with prefix x tree rows, the GEMMs with tree rows), and results travel as
  fixed-size int64 records in one ``all_gather`` (NCCL on GPUs, gloo on CPUs).
* Sequence-sharded split-KV for one long prefix.  The prefix keys are split into
  contiguous, 128-key-aligned shards; the last rank also owns the tree rows (so it is the
  rank that runs the compaction).  Every rank computes one partial (O, m, l) per row over
  its keys with ``ddt_tree_attn_partial_merged`` (the shard's tiles spread over all SMs and
  merged in-GPU).  The partials then travel over NVLink peer memory (``PeerExchange``: every
  rank stores its partial straight into every rank's receive buffer and bumps a counter
  there; each rank waits for all counters and merges) or, without one, in an NCCL
  all-gather straight into the merge layout; ``ddt_attn_merge`` gives every rank the full
  attention output.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

MAX_PATH = 21          # root + one node per drafted depth (DDT_MAX_DEPTH = 20)
RECORD_LEN = 6 + MAX_PATH


@dataclass(frozen=True)
class RequestSpec:
    index: int
    prefix: int
    budget: int
    seed: int


def request_specs(n: int = 64, seed: int = 0, lo: int = 1024, hi: int = 32768,
                  budgets=(64, 128, 256, 512)) -> list[RequestSpec]:
    """Seeded request mix: prefix lengths log-uniform in [lo, hi], budgets uniform over
    `budgets`, one drafter-logit seed per request."""
    rng = np.random.default_rng(seed)
    prefixes = np.exp(rng.uniform(math.log(lo), math.log(hi), n)).round().astype(np.int64)
    bud = rng.choice(np.asarray(budgets), n)
    return [RequestSpec(i, int(prefixes[i]), int(bud[i]), seed * 100003 + i) for i in range(n)]


def request_cost(spec: RequestSpec, layers: int = 36, q_heads: int = 32, head_dim: int = 128,
                 params: float = 8.2e9) -> float:
    """FLOPs of one verify step: tree attention 4 Hq D N P per layer plus 2 W N for the
    projections and lm_head (W = weight count), N = budget + 1 rows."""
    n = spec.budget + 1
    return n * (4.0 * q_heads * head_dim * spec.prefix * layers + 2.0 * params)


def assign_requests(costs, world: int) -> list[list[int]]:
    """Longest-processing-time first: requests in decreasing cost go to the least loaded
    rank (ties to the lower rank, then the lower request index).  Deterministic, so every
    rank computes the same assignment without communication."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0.0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda x: (load[x], x))
        out[r].append(i)
        load[r] += costs[i]
    return [sorted(o) for o in out]


def pack_result(index: int, n_nodes: int, accepted, next_token: int, time_ns: int = 0,
                rank: int = 0) -> torch.Tensor:
    """One int64 record: [index, rank, n_nodes, n_accepted, next_token, time_ns,
    accepted[0..MAX_PATH) padded with -1]."""
    rec = torch.full((RECORD_LEN,), -1, dtype=torch.int64)
    acc = list(accepted)
    if len(acc) > MAX_PATH:
        raise ValueError("accepted path longer than the record holds")
    rec[:6] = torch.tensor([index, rank, n_nodes, len(acc), next_token, time_ns])
    if acc:
        rec[6:6 + len(acc)] = torch.tensor(acc, dtype=torch.int64)
    return rec


def unpack_result(rec: torch.Tensor) -> dict:
    r = rec.tolist()
    k = r[3]
    return dict(index=r[0], rank=r[1], n_nodes=r[2], n_accepted=k, next_token=r[4], time_ns=r[5],
                accepted=r[6:6 + k])


def gather_results(records: torch.Tensor, group=None) -> torch.Tensor:
    """All-gathers variable numbers of [k, RECORD_LEN] records from every rank; returns all
    records sorted by request index (identical on every rank).  Works on NCCL (CUDA tensors)
    and gloo (CPU tensors)."""
    if not dist.is_initialized():
        return records[records[:, 0].argsort()]
    world = dist.get_world_size(group)
    dev = records.device
    cnt = torch.tensor([records.shape[0]], dtype=torch.int64, device=dev)
    counts = [torch.zeros_like(cnt) for _ in range(world)]
    dist.all_gather(counts, cnt, group=group)
    mx = int(max(c.item() for c in counts))
    pad = torch.full((mx, RECORD_LEN), -1, dtype=torch.int64, device=dev)
    pad[:records.shape[0]] = records
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    allr = torch.cat([b[:int(c.item())] for b, c in zip(bufs, counts)])
    return allr[allr[:, 0].argsort()]


def shard_range(prefix: int, n_nodes: int, world: int, rank: int, align: int = 128):
    """Global key range [begin, end) of `rank`: the prefix [0, prefix) split into
    `align`-aligned contiguous shards, the last rank also owning the tree keys
    [prefix, prefix + n_nodes).  Shards are non-empty as long as prefix >= world * align."""
    per = -(-prefix // world)
    per = -(-per // align) * align
    begin = min(rank * per, prefix)
    end = min((rank + 1) * per, prefix)
    if rank == world - 1:
        end = prefix + n_nodes
    return begin, end


def owner_rank(world: int) -> int:
    """The rank that holds the tree rows (and compacts them)."""
    return world - 1


def compact_owner_shard(keep, kv_table, shard: tuple[int, int], past_length: int) -> None:
    """KV compaction of a split-KV request (ddtree.py:284-335) on the rank that owns the tree
    keys: global rows past_length + keep[j] move to past_length + j inside this rank's shard
    [key_begin, key_end), whose K / V tensors are kv_table (local row r holds global key
    key_begin + r).  The other ranks hold prefix keys only, which compaction never moves.
    Raises ValueError on a rank whose shard does not hold the tree window."""
    from . import kernels as K
    key_begin, key_end = int(shard[0]), int(shard[1])
    keep_list = keep.tolist() if isinstance(keep, torch.Tensor) else [int(x) for x in keep]
    if not keep_list:
        return
    if not (key_begin <= past_length and past_length + max(keep_list) < key_end):
        raise ValueError(f"shard [{key_begin}, {key_end}) does not own the tree keys at "
                         f"{past_length}: compaction runs on the owner rank")
    K.compact_kv(keep if isinstance(keep, torch.Tensor) else keep_list, kv_table,
                 past_length - key_begin)


def exchange_partials(o: torch.Tensor, m: torch.Tensor, l: torch.Tensor, group=None):
    """All-gathers this rank's partials (O [S, rows, D], m [S, rows], l [S, rows]; a single
    partial may drop the leading S) into ([world * S, rows, D], [world * S, rows] x 2).
    Every rank must hold the same S."""
    if o.dim() == 2:
        o, m, l = o[None], m[None], l[None]
    if not dist.is_initialized():
        return o, m, l
    world = dist.get_world_size(group)
    s, rows, d = o.shape
    packed = torch.cat([o.reshape(-1), m.reshape(-1), l.reshape(-1)])
    bufs = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(bufs, packed, group=group)
    allp = torch.stack(bufs)
    og = allp[:, :s * rows * d].reshape(world * s, rows, d)
    mg = allp[:, s * rows * d:s * rows * (d + 1)].reshape(world * s, rows)
    lg = allp[:, s * rows * (d + 1):].reshape(world * s, rows)
    return og, mg, lg


def gather_partials(o: torch.Tensor, m: torch.Tensor, l: torch.Tensor, group=None):
    """All-gathers one partial per row and rank (O [rows, D], m [rows], l [rows]) straight
    into contiguous [world, rows, D] / [world, rows] tensors, the layout ddt_attn_merge
    reads (no packing copies)."""
    if not dist.is_initialized():
        return o[None], m[None], l[None]
    world = dist.get_world_size(group)
    out = []
    for t in (o, m, l):
        # gathered as the concatenation along dim 0 (the form every backend accepts), which
        # is the [world, ...] stack in memory
        g = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(g, t.contiguous(), group=group)
        out.append(g.view((world,) + tuple(t.shape)))
    return tuple(out)


class PeerExchange:
    """Receive buffers in NVLink peer memory for the split-KV partials of ``n_nodes`` tree
    rows x ``q_heads`` heads, one per rank of ``group`` (all on one node, at most 8), opened by
    every other rank through CUDA IPC handles that travel over the process group.

    ``exchange_merge(o, m, l)`` pushes this rank's partial into every rank's buffer
    (ddt_peer_push: 16-byte stores over NVLink, then one counter increment per buffer) and
    merges the world partials of its own buffer once every rank's push has landed
    (ddt_peer_merge, a bounded wait).  Every rank makes the same calls in the same order.
    Without an initialised process group the world is this one rank."""

    def __init__(self, n_nodes: int, q_heads: int, device, head_dim: int = 128, group=None,
                 timeout_ns: int = 2_000_000_000):
        from . import _lib
        from . import kernels as K
        self._lib = _lib.load()
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_nodes, self.q_heads, self.head_dim = n_nodes, q_heads, head_dim
        self.timeout_ns = int(timeout_ns)
        nbytes = self._lib.ddt_peer_buffer_bytes(self.world, n_nodes, q_heads, head_dim)
        if nbytes == 0:
            raise ValueError("peer exchange: unsupported world size or shape")
        with torch.cuda.device(self.device):
            ptr = ctypes.c_void_p()
            handle = (ctypes.c_char * 64)()
            _lib.check(self._lib.ddt_peer_alloc(nbytes, ctypes.byref(ptr), handle),
                       "ddt_peer_alloc")
            self.local = ptr.value
            handles = [bytes(handle)]
            if self.world > 1:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(handle), group=group)
            self.peers, self._opened = [], []
            try:
                for r in range(self.world):
                    if r == self.rank:
                        self.peers.append(self.local)
                        continue
                    pp = ctypes.c_void_p()
                    buf = (ctypes.c_char * 64).from_buffer_copy(handles[r])
                    _lib.check(self._lib.ddt_peer_open(buf, ctypes.byref(pp)), "ddt_peer_open")
                    self.peers.append(pp.value)
                    self._opened.append(pp.value)
            except Exception:
                self.close()
                raise
        self._bases = (ctypes.c_void_p * self.world)(*self.peers)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.status = K.attention_status(self.device)
        self.epoch = 0
        if self.world > 1:
            dist.barrier(group=group)  # every buffer is open before the first push

    def exchange_merge(self, o: torch.Tensor, m: torch.Tensor, l: torch.Tensor,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        from . import kernels as K
        from ._lib import check
        n, hq, d = self.n_nodes, self.q_heads, self.head_dim
        if out is None:
            out = torch.empty((n, hq, d), dtype=torch.bfloat16, device=self.device)
        o, m, l = o.contiguous(), m.contiguous(), l.contiguous()
        self.epoch += 1
        st = torch.cuda.current_stream(self.device).cuda_stream
        check(self._lib.ddt_peer_push(o.data_ptr(), m.data_ptr(), l.data_ptr(), n, hq, d,
                                      ctypes.cast(self._bases, ctypes.c_void_p), self.world,
                                      self.rank, self.epoch & 0xffffffff, self.ticket.data_ptr(),
                                      st), "ddt_peer_push")
        check(self._lib.ddt_peer_merge(self.local, self.world, n, hq, d, self.epoch & 0xffffffff,
                                       out.data_ptr(), out.stride(0), out.stride(1),
                                       self.status.data_ptr(), self.timeout_ns, st),
              "ddt_peer_merge")
        K.STATS.launches += 3
        return out

    def attend(self, q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
               key_begin: int, key_end: int, anc_bits: torch.Tensor | None, past_length: int,
               scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's shard attention whose merge stores the partial straight into every
        rank's buffer (ddt_tree_attn_partial_push, one call), then the counter-waiting merge
        of all ranks' partials (ddt_peer_merge).  Returns the bf16 output [N, Hq, D]."""
        self.attend_push(q, k_shard, v_shard, key_begin, key_end, anc_bits, past_length, scale)
        return self.merge(out)

    def attend_push(self, q, k_shard, v_shard, key_begin: int, key_end: int, anc_bits,
                    past_length: int, scale: float | None = None) -> None:
        """The first half of attend: shard attention + push of this call's partial."""
        from . import kernels as K
        from ._lib import DDT_MASK_TREE, check
        n, hq, qns, qhs = K._q_view(q)
        hkv, s_local, khs, kss = K._kv_view(k_shard)
        d = q.shape[-1]
        if (n, hq, d) != (self.n_nodes, self.q_heads, self.head_dim):
            raise ValueError("query shape differs from the exchange's")
        if s_local < key_end - key_begin:
            raise ValueError("shard shorter than its key range")
        if scale is None:
            scale = 1.0 / math.sqrt(d)
        ws_bytes = self._lib.ddt_tree_attn_partial_push_workspace_bytes(n, hq, d)
        ws = K.WORKSPACES.get(self.device, "attn_partial_push", ws_bytes)
        words = anc_bits.shape[1] if anc_bits is not None else 0
        self.epoch += 1
        st = torch.cuda.current_stream(self.device).cuda_stream
        check(self._lib.ddt_tree_attn_partial_push(
            q.data_ptr(), qns, qhs, k_shard.data_ptr(), v_shard.data_ptr(), khs, kss, key_begin,
            key_end, n, past_length, hq, hkv, d,
            anc_bits.data_ptr() if anc_bits is not None else None, words, DDT_MASK_TREE,
            float(scale), ctypes.cast(self._bases, ctypes.c_void_p), self.world, self.rank,
            self.epoch & 0xffffffff, self.ticket.data_ptr(), ws.data_ptr(), ws.numel(),
            self.status.data_ptr(), st), "ddt_tree_attn_partial_push")
        K.STATS.launches += 2

    def merge(self, out: torch.Tensor | None = None) -> torch.Tensor:
        """The second half of attend: wait for every rank's push of the current call, merge."""
        from . import kernels as K
        from ._lib import check
        n, hq, d = self.n_nodes, self.q_heads, self.head_dim
        if out is None:
            out = torch.empty((n, hq, d), dtype=torch.bfloat16, device=self.device)
        st = torch.cuda.current_stream(self.device).cuda_stream
        check(self._lib.ddt_peer_merge(self.local, self.world, n, hq, d, self.epoch & 0xffffffff,
                                       out.data_ptr(), out.stride(0), out.stride(1),
                                       self.status.data_ptr(), self.timeout_ns, st),
              "ddt_peer_merge")
        K.STATS.launches += 2
        return out

    def close(self) -> None:
        """Releases the IPC mappings and the buffer (after a barrier, so that no peer still
        writes into it)."""
        if getattr(self, "local", None) is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1 and dist.is_initialized():
            dist.barrier(group=self.group)
        for p in getattr(self, "_opened", []):
            self._lib.ddt_peer_close(ctypes.c_void_p(p))
        self._opened = []
        self._lib.ddt_peer_free(ctypes.c_void_p(self.local))
        self.local = None


def splitkv_attention(q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                      key_begin: int, key_end: int, anc_bits: torch.Tensor | None,
                      past_length: int, scale: float | None = None, group=None,
                      out: torch.Tensor | None = None,
                      exchange: PeerExchange | None = None) -> torch.Tensor:
    """Tree attention over a sequence-sharded prefix: this rank's keys spread over all of its
    SMs and merged in-GPU to one partial per row, the partials of all ranks exchanged, merge.
    With ``exchange`` the in-GPU merge itself stores the partial into every rank's buffer over
    NVLink (PeerExchange.attend); without, one NCCL all-gather.  Returns the bf16 output
    [N, Hq, D] on every rank."""
    from . import kernels as K
    n, hq = q.shape[0], q.shape[1]
    if exchange is not None:
        return exchange.attend(q, k_shard, v_shard, key_begin, key_end, anc_bits, past_length,
                               scale=scale, out=out)
    o, m, l = K.tree_attention_partial_merged(q, k_shard, v_shard, key_begin, key_end, anc_bits,
                                              past_length, scale=scale)
    og, mg, lg = gather_partials(o, m, l, group)
    return K.attn_merge(og, mg, lg, n, hq, out=out)
