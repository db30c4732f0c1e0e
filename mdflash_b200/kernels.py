"""Tensor-level wrappers over the C ABI.  PyTorch owns every buffer; the kernels run on
the current CUDA stream of the tensors' device and never synchronise the host."""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import DDT_BF16, DDT_F32, DDT_MASK_CAUSAL, DDT_MASK_NONE, DDT_MASK_TREE, check

__all__ = [
    "DeviceTree", "expected_node_count", "topk_tree", "argmax", "accept_compact", "compact_kv",
    "tree_attention", "tree_attention_partial", "attn_merge", "mask_to_bits", "KvTable",
    "anc_words_for", "TreeBatch", "topk_tree_batched", "KvBatch", "accept_compact_batched",
    "attention_status", "check_status", "tree_attention_wait_check",
    "sample_chains", "chain_tree", "lm_head_argmax",
]


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class LaunchStats:
    """Counts this library's kernel launches, and (when enabled) brackets every tree
    attention call with CUDA events on its stream so its device time can be measured
    inside a larger timed region."""

    def __init__(self):
        self.launches = 0
        self.time_attention = False
        self.attn_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []

    def reset(self, time_attention: bool = False) -> None:
        self.launches = 0
        self.time_attention = time_attention
        self.attn_events = []

    def attention_ms(self) -> list[float]:
        return [a.elapsed_time(b) for a, b in self.attn_events]


STATS = LaunchStats()


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return DDT_BF16
    if t.dtype == torch.float32:
        return DDT_F32
    raise TypeError(f"unsupported dtype {t.dtype}")


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if not t.is_cuda:
            raise ValueError("ddtree_b200 kernels need CUDA tensors")
        if t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


class _Workspaces:
    """Per-device scratch buffers, grown on demand and zero-filled when (re)allocated.

    A buffer that is outgrown is kept alive, not freed: CUDA graphs captured earlier still
    hold its address, and freed memory could be handed to another tensor.  Buffers are also
    keyed by the current lane (``lane``): graphs that may replay concurrently on different
    streams are captured in different lanes, so they share no scratch."""

    def __init__(self):
        self._bufs: dict[tuple[int, str, int], torch.Tensor] = {}
        self._retired: list[torch.Tensor] = []
        self.current_lane = 0

    def get(self, device: torch.device, name: str, nbytes: int) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        key = (idx, name, self.current_lane)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            nb = max(nbytes, 256)
            if buf is not None:
                nb = max(nb, 2 * buf.numel())
                self._retired.append(buf)
            buf = torch.zeros(nb, dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf

    @contextlib.contextmanager
    def lane(self, lane: int):
        prev, self.current_lane = self.current_lane, int(lane)
        try:
            yield
        finally:
            self.current_lane = prev


WORKSPACES = _Workspaces()


def attention_status(device: torch.device) -> torch.Tensor:
    """The device's default status word (i32 [1]) of tree-attention launches that are given
    none: a bounded wait of the kernel that ran out sets it non-zero."""
    with WORKSPACES.lane(0):  # one status word per device, whatever lane a launch runs in
        return WORKSPACES.get(device, "attn_status", 256)[:4].view(torch.int32)


STATUS_TIMEOUT = 1      # a bounded wait of a kernel ran out
STATUS_LAYOUT = 2       # a batched compaction met a head stride it cannot move
STATUS_PAST_RANGE = 4   # a device-side prefix length was outside [0, planned maximum]
STATUS_LOG_FULL = 8     # a decode-loop round found its output or length log full


def check_status(status: torch.Tensor, what: str = "ddt_tree_attn") -> None:
    """Reads a status word (this syncs with its stream) and raises DDTreeError when a launch
    that wrote to it reported an error: DDT_ERR_TIMEOUT when a bounded wait ran out,
    DDT_ERR_INVALID for a device-side prefix length out of range or a layout the batched
    compaction cannot move.  The word is cleared first, so the next launches start clean."""
    v = int(status.reshape(-1)[0].item())
    if v != 0:
        status.zero_()
        if v & STATUS_TIMEOUT:
            check(_lib.DDT_ERR_TIMEOUT, what)
        why = ("prefix length out of range" if v & STATUS_PAST_RANGE else
               "decode-loop log full" if v & STATUS_LOG_FULL else "invalid KV layout")
        raise _lib.DDTreeError(f"{what}: device status {v:#x} ({why})")


def anc_words_for(n_nodes: int) -> int:
    return max(1, (n_nodes + 31) // 32)


def expected_node_count(depths: int, vocab: int, budget: int) -> int:
    """Nodes (without the root) the best-first expansion produces: the budget, unless
    the whole tree of sum_{d=1..depths} k^d candidates is smaller (k = min(budget, V))."""
    if budget <= 0 or depths <= 0:
        return 0
    k = min(budget, vocab)
    total = 0
    for d in range(1, depths + 1):
        total += k ** d
        if total >= budget:
            return budget
    return min(budget, total)


@dataclass
class DeviceTree:
    """Device-resident draft tree (node 0 is the root)."""
    budget: int
    depths: int
    k: int
    n_nodes: int                   # 1 + node count, known on the host without a sync
    node_count: torch.Tensor       # i32 [1]
    node_token_ids: torch.Tensor   # i64 [budget]
    node_depths: torch.Tensor      # i64 [budget]
    parents: torch.Tensor          # i32 [budget + 1]
    anc_bits: torch.Tensor         # i32 (bit pattern of u32) [budget + 1, anc_words]
    verify_ids: torch.Tensor       # i64 [budget + 1]
    verify_pos: torch.Tensor       # i64 [budget + 1]
    top_log_probs: torch.Tensor    # f32 [depths, k]
    top_token_ids: torch.Tensor    # i64 [depths, k]

    @property
    def anc_words(self) -> int:
        return self.anc_bits.shape[1]

    @staticmethod
    def allocate(device, budget: int, depths: int, vocab: int) -> "DeviceTree":
        b = max(budget, 0)
        k = min(b, vocab) if b > 0 else 0
        n_cap = b + 1
        i64 = dict(dtype=torch.int64, device=device)
        return DeviceTree(
            budget=b, depths=depths, k=k, n_nodes=1 + expected_node_count(depths, vocab, b),
            node_count=torch.zeros(1, dtype=torch.int32, device=device),
            node_token_ids=torch.zeros(max(b, 1), **i64),
            node_depths=torch.zeros(max(b, 1), **i64),
            parents=torch.zeros(n_cap, dtype=torch.int32, device=device),
            anc_bits=torch.zeros((n_cap, anc_words_for(n_cap)), dtype=torch.int32, device=device),
            verify_ids=torch.zeros(n_cap, **i64), verify_pos=torch.zeros(n_cap, **i64),
            top_log_probs=torch.zeros((max(depths, 1), max(k, 1)), dtype=torch.float32,
                                      device=device),
            top_token_ids=torch.zeros((max(depths, 1), max(k, 1)), **i64))


def topk_tree(draft_logits: torch.Tensor, budget: int, root_token: torch.Tensor | None = None,
              start: int = 0, out: DeviceTree | None = None) -> DeviceTree:
    """Per-depth log Z + top-k, best-first tree, ancestor bitmasks and verify ids /
    positions in one launch (ddtree.py:84-166 and :248-257)."""
    if draft_logits.dim() != 2:
        raise ValueError("draft_logits must be [depths, vocab]")
    dev = _require_cuda(draft_logits)
    L, V = draft_logits.shape
    if draft_logits.stride(1) != 1:
        draft_logits = draft_logits.contiguous()
    tree = out if out is not None else DeviceTree.allocate(dev, budget, L, V)
    if tree.budget != max(budget, 0) or tree.depths != L:
        raise ValueError("output DeviceTree was allocated for another budget / depth")
    tree.n_nodes = 1 + expected_node_count(L, V, budget)
    lib = _lib.load()
    ws_bytes = lib.ddt_topk_tree_workspace_bytes(L, V, budget)
    ws = WORKSPACES.get(dev, "topk_tree", ws_bytes)
    if root_token is not None:
        root_token = root_token.reshape(-1)[:1]
        if root_token.dtype != torch.int64:
            root_token = root_token.to(torch.int64)
    rc = lib.ddt_topk_tree(
        draft_logits.data_ptr(), _dtype_code(draft_logits), L, V, draft_logits.stride(0), budget,
        tree.top_log_probs.data_ptr(), tree.top_token_ids.data_ptr(), tree.node_token_ids.data_ptr(),
        tree.node_depths.data_ptr(), tree.parents.data_ptr(), tree.node_count.data_ptr(),
        tree.anc_bits.data_ptr(), tree.anc_words,
        root_token.data_ptr() if root_token is not None else None, int(start),
        tree.verify_ids.data_ptr(), tree.verify_pos.data_ptr(), ws.data_ptr(), ws.numel(),
        _stream(dev))
    check(rc, "ddt_topk_tree")
    STATS.launches += 1
    return tree


@dataclass
class TreeBatch:
    """The trees of a batched build (ddt_topk_tree_batched): request r's outputs are row r of
    each [n_requests, ...] tensor; ``tree(r)`` views them as a DeviceTree."""
    budgets: list[int]             # per request (host copy; the device copy is budgets_dev)
    max_budget: int
    depths: int
    vocab: int
    budgets_dev: torch.Tensor      # i32 [R]
    starts: torch.Tensor           # i64 [R]
    root_tokens: torch.Tensor      # i64 [R]
    node_count: torch.Tensor       # i32 [R]
    node_token_ids: torch.Tensor   # i64 [R, max_budget]
    node_depths: torch.Tensor      # i64 [R, max_budget]
    parents: torch.Tensor          # i32 [R, max_budget + 1]
    anc_bits: torch.Tensor         # i32 [R, max_budget + 1, anc_words]
    verify_ids: torch.Tensor       # i64 [R, max_budget + 1]
    verify_pos: torch.Tensor       # i64 [R, max_budget + 1]

    @staticmethod
    def allocate(device, budgets: list[int], depths: int, vocab: int) -> "TreeBatch":
        R = len(budgets)
        mb = max([max(int(b), 0) for b in budgets] + [1])
        i64 = dict(dtype=torch.int64, device=device)
        return TreeBatch(
            budgets=[max(int(b), 0) for b in budgets], max_budget=mb, depths=depths, vocab=vocab,
            budgets_dev=torch.tensor([max(int(b), 0) for b in budgets], dtype=torch.int32,
                                     device=device),
            starts=torch.zeros(R, **i64), root_tokens=torch.zeros(R, **i64),
            node_count=torch.zeros(R, dtype=torch.int32, device=device),
            node_token_ids=torch.zeros((R, mb), **i64), node_depths=torch.zeros((R, mb), **i64),
            parents=torch.zeros((R, mb + 1), dtype=torch.int32, device=device),
            anc_bits=torch.zeros((R, mb + 1, anc_words_for(mb + 1)), dtype=torch.int32,
                                 device=device),
            verify_ids=torch.zeros((R, mb + 1), **i64), verify_pos=torch.zeros((R, mb + 1), **i64))

    def tree(self, r: int) -> DeviceTree:
        b = self.budgets[r]
        k = min(b, self.vocab) if b > 0 else 0
        dev = self.parents.device
        return DeviceTree(
            budget=b, depths=self.depths, k=k,
            n_nodes=1 + expected_node_count(self.depths, self.vocab, b),
            node_count=self.node_count[r:r + 1], node_token_ids=self.node_token_ids[r, :max(b, 1)],
            node_depths=self.node_depths[r, :max(b, 1)], parents=self.parents[r, :b + 1],
            anc_bits=self.anc_bits[r, :b + 1], verify_ids=self.verify_ids[r, :b + 1],
            verify_pos=self.verify_pos[r, :b + 1],
            # the batched build keeps no per-depth top-k tables
            top_log_probs=torch.zeros((max(self.depths, 1), 0), dtype=torch.float32, device=dev),
            top_token_ids=torch.zeros((max(self.depths, 1), 0), dtype=torch.int64, device=dev))


def topk_tree_batched(draft_logits: torch.Tensor, out: TreeBatch) -> TreeBatch:
    """ddt_topk_tree_batched: the tree of every request of ``draft_logits`` [R, depths, vocab]
    in one launch, with out.budgets_dev, out.root_tokens and out.starts as inputs (fill them
    before the call); request r's tree equals topk_tree(draft_logits[r], budgets[r],
    root_tokens[r], starts[r])."""
    if draft_logits.dim() != 3:
        raise ValueError("draft_logits must be [requests, depths, vocab]")
    dev = _require_cuda(draft_logits)
    R, L, V = draft_logits.shape
    if draft_logits.stride(2) != 1:
        draft_logits = draft_logits.contiguous()
    if R != len(out.budgets) or L != out.depths or V != out.vocab:
        raise ValueError("TreeBatch was allocated for another request count / depth / vocabulary")
    lib = _lib.load()
    ws_bytes = lib.ddt_topk_tree_batched_workspace_bytes(R, L, V, out.max_budget)
    ws = WORKSPACES.get(dev, "topk_tree_batched", ws_bytes)
    check(lib.ddt_topk_tree_batched(
        draft_logits.data_ptr(), _dtype_code(draft_logits), R, L, V, draft_logits.stride(1),
        draft_logits.stride(0), out.budgets_dev.data_ptr(), out.max_budget,
        out.node_token_ids.data_ptr(), out.node_depths.data_ptr(), out.parents.data_ptr(),
        out.node_count.data_ptr(), out.anc_bits.data_ptr(), out.anc_bits.shape[2],
        out.root_tokens.data_ptr(), out.starts.data_ptr(), out.verify_ids.data_ptr(),
        out.verify_pos.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev)),
        "ddt_topk_tree_batched")
    STATS.launches += 1
    return out


def sample_chains(draft_logits: torch.Tensor, num_samples: int, temperature: float, seed: int,
                  offset: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """ddt_sample_chains: i64 [num_samples, depths] chains, sample s of every depth drawn
    from softmax(draft_logits / temperature) (argmax for temperature < 1e-5)."""
    if draft_logits.dim() != 2:
        raise ValueError("draft_logits must be [depths, vocab]")
    dev = _require_cuda(draft_logits)
    L, V = draft_logits.shape
    if draft_logits.stride(1) != 1:
        draft_logits = draft_logits.contiguous()
    if out is None:
        out = torch.empty((max(num_samples, 0), L), dtype=torch.int64, device=dev)
    check(_lib.load().ddt_sample_chains(
        draft_logits.data_ptr(), _dtype_code(draft_logits), L, V, draft_logits.stride(0),
        num_samples, float(temperature), int(seed) & ((1 << 64) - 1),
        int(offset) & ((1 << 64) - 1), out.data_ptr(), _stream(dev)), "ddt_sample_chains")
    STATS.launches += 1
    return out


def chain_tree(chains: torch.Tensor, budget: int, root_token: torch.Tensor | None = None,
               start: int = 0, out: DeviceTree | None = None) -> DeviceTree:
    """ddt_chain_tree: the trie of i64 [num_chains, depths] chains with at most `budget`
    nodes (ddtree.py:169-224), as a DeviceTree.  Its node count is data-dependent:
    tree.n_nodes is set to 1 + budget (an upper bound); tree.node_count holds the count."""
    if chains.dim() != 2:
        raise ValueError("chains must be [num_chains, depths]")
    dev = _require_cuda(chains)
    S, L = chains.shape
    if chains.dtype != torch.int64:
        chains = chains.to(torch.int64)
    if chains.stride(1) != 1:
        chains = chains.contiguous()
    b = max(int(budget), 0)
    tree = out if out is not None else DeviceTree.allocate(dev, b, max(L, 1), b if b > 0 else 1)
    if tree.budget != b:
        raise ValueError("output DeviceTree was allocated for another budget")
    tree.n_nodes = 1 + b
    if root_token is not None:
        root_token = root_token.reshape(-1)[:1]
        if root_token.dtype != torch.int64:
            root_token = root_token.to(torch.int64)
    check(_lib.load().ddt_chain_tree(
        chains.data_ptr() if chains.numel() else None, S, L, max(chains.stride(0), L), b,
        tree.node_token_ids.data_ptr(), tree.node_depths.data_ptr(), tree.parents.data_ptr(),
        tree.node_count.data_ptr(), tree.anc_bits.data_ptr(), tree.anc_words,
        root_token.data_ptr() if root_token is not None else None, int(start),
        tree.verify_ids.data_ptr(), tree.verify_pos.data_ptr(), _stream(dev)), "ddt_chain_tree")
    STATS.launches += 1
    return tree


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Row argmax over the last dim (lowest index on ties, NaN largest)."""
    dev = _require_cuda(logits)
    x = logits.reshape(-1, logits.shape[-1])
    if x.stride(1) != 1:
        x = x.contiguous()
    rows, cols = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=dev)
    check(_lib.load().ddt_argmax(x.data_ptr(), _dtype_code(x), rows, cols, x.stride(0),
                                 out.data_ptr(), _stream(dev)), "ddt_argmax")
    STATS.launches += 1
    return out.view(logits.shape[:-1])


def lm_head_argmax(hidden: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None,
                   logits_out: torch.Tensor | None = None,
                   status: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy posterior of the lm_head without materialising the logits: out[n] =
    argmax_v bf16(hidden[n] . weight[v]) (ties to the lowest index).  hidden [N, H] and
    weight [V, H] bf16 with unit inner stride; logits_out ([N, V] bf16), when given, receives
    the bf16 logits the argmax was taken over."""
    dev = _require_cuda(hidden, weight)
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("lm_head_argmax takes bf16 hidden states and weight")
    h = hidden.reshape(-1, hidden.shape[-1])
    if h.stride(1) != 1:
        h = h.contiguous()
    if weight.stride(1) != 1:
        raise ValueError("weight rows must be contiguous")
    n, H = h.shape
    V = weight.shape[0]
    if out is None:
        out = torch.empty(n, dtype=torch.int64, device=dev)
    if status is None:
        status = attention_status(dev)
    lib = _lib.load()
    ws = WORKSPACES.get(dev, "lm_head_argmax", lib.ddt_lm_head_argmax_workspace_bytes(n))
    lo_ptr, lo_ld = (None, 0) if logits_out is None else (logits_out.data_ptr(),
                                                         logits_out.stride(0))
    check(lib.ddt_lm_head_argmax(h.data_ptr(), h.stride(0), weight.data_ptr(), weight.stride(0),
                                 n, H, V, out.data_ptr(), lo_ptr, lo_ld, ws.data_ptr(), ws.numel(),
                                 status.data_ptr(), _stream(dev)), "ddt_lm_head_argmax")
    STATS.launches += 1
    return out


class KvTable:
    """Device table of K/V base pointers ([heads, seq, head_dim] views, head_dim
    contiguous, identical strides) for the one-launch compaction kernels."""

    def __init__(self, tensors: list[torch.Tensor]):
        if not tensors:
            raise ValueError("empty KV table")
        t0 = tensors[0]
        self.device = _require_cuda(*tensors)
        if t0.dim() == 4:
            if t0.shape[0] != 1:
                raise ValueError("batch size 1 caches only")
            tensors = [t[0] for t in tensors]
            t0 = tensors[0]
        self.heads, self.seq, self.head_dim = t0.shape
        self.head_stride, self.seq_stride, inner = t0.stride()
        for t in tensors:
            if t.shape[0] != self.heads or t.shape[2] != self.head_dim or \
                    t.stride() != (self.head_stride, self.seq_stride, 1) or t.dtype != t0.dtype:
                raise ValueError("KV tensors must share shape, strides and dtype")
        if inner != 1:
            raise ValueError("head_dim must be contiguous")
        self.elem_bytes = t0.element_size()
        self.n = len(tensors)
        self.ptrs = torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64,
                                 device=self.device)
        self._keep = tensors  # keep storages alive


def accept_compact(posterior: torch.Tensor, tree: DeviceTree, kv: KvTable, past_length: int,
                   accepted: torch.Tensor | None = None, n_accepted: torch.Tensor | None = None,
                   next_token: torch.Tensor | None = None, n_nodes: int | None = None):
    """Greedy accept walk + KV compaction in one launch (ddtree.py:270-281, 284-335)."""
    dev = _require_cuda(posterior)
    n = tree.n_nodes if n_nodes is None else n_nodes
    if past_length + n > kv.seq:
        raise ValueError(f"cache holds {kv.seq} rows, the tree window needs {past_length + n}")
    if accepted is None:
        accepted = torch.zeros(n, dtype=torch.int64, device=dev)
    if n_accepted is None:
        n_accepted = torch.zeros(1, dtype=torch.int32, device=dev)
    if next_token is None:
        next_token = torch.zeros(1, dtype=torch.int64, device=dev)
    post = posterior.reshape(-1)
    if post.dtype != torch.int64:
        post = post.to(torch.int64)
    check(_lib.load().ddt_accept_compact(
        post.data_ptr(), tree.parents.data_ptr(), tree.node_token_ids.data_ptr(), n,
        kv.ptrs.data_ptr(), kv.n, kv.heads, kv.head_dim, kv.head_stride, kv.seq_stride,
        kv.elem_bytes, past_length, accepted.data_ptr(), n_accepted.data_ptr(),
        next_token.data_ptr(), _stream(dev)), "ddt_accept_compact")
    STATS.launches += 1
    return accepted, n_accepted, next_token


class KvBatch:
    """The K/V tables of several requests for the batched walk + compaction: the tables share
    tensor count, heads, head_dim, sequence stride and dtype; their capacities (head strides)
    may differ."""

    def __init__(self, tables: list[KvTable]):
        if not tables:
            raise ValueError("empty KV batch")
        t0 = tables[0]
        for t in tables:
            if (t.n, t.heads, t.head_dim, t.seq_stride, t.elem_bytes) != \
                    (t0.n, t0.heads, t0.head_dim, t0.seq_stride, t0.elem_bytes):
                raise ValueError("KV tables of a batch must share layout and dtype")
        self.tables = tables
        self.device = t0.device
        self.n, self.heads, self.head_dim = t0.n, t0.heads, t0.head_dim
        self.seq_stride, self.elem_bytes = t0.seq_stride, t0.elem_bytes
        self.capacity = [t.seq for t in tables]
        self.ptrs = torch.cat([t.ptrs for t in tables])
        self.head_strides = torch.tensor([t.head_stride for t in tables], dtype=torch.int64,
                                         device=self.device)


def accept_compact_batched(posteriors: torch.Tensor, trees: TreeBatch, kvb: KvBatch,
                           past_lengths, accepted: torch.Tensor | None = None,
                           n_accepted: torch.Tensor | None = None,
                           next_token: torch.Tensor | None = None,
                           status: torch.Tensor | None = None):
    """ddt_accept_compact_batched: the greedy walk of every request's tree (trees, one row per
    request) under its posterior row (posteriors [R, max_budget + 1] i64) and the compaction of
    its cache.  past_lengths: a host list (checked against every cache's capacity) or a device
    i64 tensor (trusted, no host work per call).  Returns (accepted [R, max_budget + 1],
    n_accepted i32 [R], next_token i64 [R])."""
    dev = _require_cuda(posteriors)
    R = len(trees.budgets)
    mn = trees.max_budget + 1
    if posteriors.shape != (R, mn) or posteriors.dtype != torch.int64 or posteriors.stride(1) != 1:
        raise ValueError("posteriors must be i64 [requests, max_budget + 1] with unit stride")
    if len(kvb.tables) != R:
        raise ValueError("one KV table per request")
    if isinstance(past_lengths, torch.Tensor) and past_lengths.is_cuda:
        if past_lengths.dtype != torch.int64 or past_lengths.numel() != R:
            raise ValueError("past_lengths must be i64 [requests]")
        past_dev = past_lengths.contiguous()
    else:
        past = [int(x) for x in past_lengths]
        for r in range(R):
            n = 1 + expected_node_count(trees.depths, trees.vocab, trees.budgets[r])
            if past[r] < 0 or past[r] + n > kvb.capacity[r]:
                raise ValueError(f"request {r}: cache holds {kvb.capacity[r]} rows, the tree "
                                 f"window needs {past[r] + n}")
        past_dev = torch.tensor(past, dtype=torch.int64, device=dev)
    if accepted is None:
        accepted = torch.zeros((R, mn), dtype=torch.int64, device=dev)
    if n_accepted is None:
        n_accepted = torch.zeros(R, dtype=torch.int32, device=dev)
    if next_token is None:
        next_token = torch.zeros(R, dtype=torch.int64, device=dev)
    if status is None:
        status = attention_status(dev)
    check(_lib.load().ddt_accept_compact_batched(
        R, posteriors.data_ptr(), posteriors.stride(0), trees.parents.data_ptr(),
        trees.parents.stride(0), trees.node_token_ids.data_ptr(), trees.node_token_ids.stride(0),
        trees.node_count.data_ptr(), mn, kvb.ptrs.data_ptr(), kvb.n, kvb.heads, kvb.head_dim,
        kvb.head_strides.data_ptr(), kvb.seq_stride, kvb.elem_bytes, past_dev.data_ptr(),
        accepted.data_ptr(), accepted.stride(0), n_accepted.data_ptr(), next_token.data_ptr(),
        status.data_ptr(), _stream(dev)), "ddt_accept_compact_batched")
    STATS.launches += 1
    return accepted, n_accepted, next_token


def advance_round(starts: torch.Tensor, rounds: torch.Tensor, n_accepted: torch.Tensor,
                  accepted: torch.Tensor, verify_ids: torch.Tensor, next_token: torch.Tensor,
                  root_tokens: torch.Tensor, output_ids: torch.Tensor, acceptance: torch.Tensor,
                  status: torch.Tensor | None = None) -> None:
    """ddt_advance_round: one decode-loop round's bookkeeping on the device for R requests
    (ddtree.py:488-498): the accepted tokens and the next token into output_ids [R, cap] at
    starts[r], the next token into root_tokens[r], n_accepted[r] into acceptance[R, rounds]
    at rounds[r]; then rounds[r] += 1 and starts[r] += n_accepted[r].  starts / root_tokens /
    next_token i64 [R], rounds / n_accepted i32 [R], accepted / verify_ids i64 [R, nodes]."""
    dev = _require_cuda(starts)
    R = starts.numel()
    for t, dt, name in ((starts, torch.int64, "starts"), (rounds, torch.int32, "rounds"),
                        (n_accepted, torch.int32, "n_accepted"),
                        (next_token, torch.int64, "next_token"),
                        (root_tokens, torch.int64, "root_tokens")):
        if t.dtype != dt or t.numel() != R or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous {dt} [{R}]")
    acc = accepted.reshape(R, -1)
    vid = verify_ids.reshape(R, -1)
    out = output_ids.reshape(R, -1)
    lens = acceptance.reshape(R, -1)
    if acc.dtype != torch.int64 or vid.dtype != torch.int64 or out.dtype != torch.int64 or \
            lens.dtype != torch.int32:
        raise ValueError("accepted / verify_ids / output_ids must be i64, acceptance i32")
    if any(t.stride(1) != 1 for t in (acc, vid, out, lens)):
        raise ValueError("rows must have unit stride")
    if status is None:
        status = attention_status(dev)
    check(_lib.load().ddt_advance_round(
        R, starts.data_ptr(), rounds.data_ptr(), n_accepted.data_ptr(), acc.data_ptr(),
        acc.stride(0), vid.data_ptr(), vid.stride(0), vid.shape[1], next_token.data_ptr(),
        root_tokens.data_ptr(), out.data_ptr(), out.stride(0), out.shape[1], lens.data_ptr(),
        lens.stride(0), lens.shape[1], status.data_ptr(), _stream(dev)), "ddt_advance_round")
    STATS.launches += 1


def gather_rows(src: torch.Tensor, idx: torch.Tensor, count: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """ddt_gather_rows: out[i] = src[idx[i]] for i < count (a device i32 [1], read on the
    device; None: every index), rows of src [rows, ...] (the row contiguous); the rows of out
    at or beyond the count keep their contents."""
    dev = _require_cuda(src, idx)
    if idx.dtype != torch.int64 or idx.dim() != 1 or not idx.is_contiguous():
        raise ValueError("idx must be a contiguous i64 vector")
    if count is not None and (count.dtype != torch.int32 or count.numel() != 1):
        raise ValueError("count must be an i32 [1]")
    rows = src.shape[0]
    row = src[0].numel() if rows else 0
    if rows and src[0].is_contiguous() is False:
        raise ValueError("src rows must be contiguous")
    if out is None:
        out = torch.zeros((idx.numel(),) + tuple(src.shape[1:]), dtype=src.dtype, device=dev)
    if out.shape[1:] != src.shape[1:] or out.dtype != src.dtype or out.shape[0] < idx.numel():
        raise ValueError("out must match src's row shape and dtype, with a row per index")
    es = src.element_size()
    check(_lib.load().ddt_gather_rows(
        src.data_ptr(), rows, src.stride(0) * es, idx.data_ptr(),
        count.data_ptr() if count is not None else None, idx.numel(), out.data_ptr(),
        out.stride(0) * es, row * es, _stream(dev)), "ddt_gather_rows")
    STATS.launches += 1
    return out


def compact_kv(keep, kv: KvTable, past_length: int) -> None:
    """Moves rows past_length + keep[j] -> past_length + j in every table tensor.  A host
    list is validated (strictly increasing, inside the cache); a device tensor is trusted."""
    if not isinstance(keep, torch.Tensor):
        keep = [int(x) for x in keep]
        if any(b <= a for a, b in zip(keep, keep[1:])) or (keep and keep[0] < 0):
            raise ValueError("keep indices must be strictly increasing and non-negative")
        if keep and past_length + keep[-1] >= kv.seq:
            raise ValueError("keep index outside the cache window")
        keep = torch.tensor(keep, dtype=torch.int64, device=kv.device)
    keep = keep.reshape(-1)
    if keep.dtype != torch.int64:
        keep = keep.to(torch.int64)
    check(_lib.load().ddt_compact_kv(keep.data_ptr(), keep.numel(), kv.ptrs.data_ptr(), kv.n,
                                     kv.heads, kv.head_dim, kv.head_stride, kv.seq_stride,
                                     kv.elem_bytes, past_length, _stream(kv.device)),
          "ddt_compact_kv")
    STATS.launches += 1


def _q_view(q: torch.Tensor):
    """Accepts [N, Hq, D] or HF's [1, Hq, N, D]; returns (N, Hq, node_stride, head_stride)."""
    if q.dim() == 4:
        if q.shape[0] != 1:
            raise ValueError("batch size 1 only")
        _, hq, n, d = q.shape
        return n, hq, q.stride(2), q.stride(1)
    n, hq, d = q.shape
    return n, hq, q.stride(0), q.stride(1)


def _kv_view(k: torch.Tensor):
    """Accepts [Hkv, S, D] or [1, Hkv, S, D]; returns (Hkv, S, head_stride, seq_stride)."""
    if k.dim() == 4:
        if k.shape[0] != 1:
            raise ValueError("batch size 1 only")
        k = k[0]
    return k.shape[0], k.shape[1], k.stride(0), k.stride(1)


def _mask_mode(causal: bool, unmasked: bool) -> int:
    if causal and unmasked:
        raise ValueError("causal and unmasked are exclusive")
    return DDT_MASK_NONE if unmasked else (DDT_MASK_CAUSAL if causal else DDT_MASK_TREE)


def tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   anc_bits: torch.Tensor | None, past_length: int, scale: float | None = None,
                   causal: bool = False, out: torch.Tensor | None = None, kv_splits: int = 0,
                   status: torch.Tensor | None = None, unmasked: bool = False,
                   past_dev: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(Q K^T * scale, tree / causal mask) V on tcgen05.  q: [N, Hq, D] (or HF
    [1, Hq, N, D]); k, v: [Hkv, past_length + N, D] (or [1, ...]); returns [N, Hq, D].
    Mask: the tree (anc_bits), causal=True (node i sees keys < past_length + i + 1), or
    unmasked=True (every row sees every key: the drafter's non-causal attention).

    past_dev (i64 [1], device): the prefix length is read from it when the kernel runs
    (ddt_tree_attn_device_past), past_length is then its maximum and k / v cover
    past_length + N rows; a recorded launch serves every prefix length up to past_length.

    The kernel computes in bf16 (fp32 accumulation).  fp32 inputs (an fp32 model) are rounded
    to bf16 for the kernel and the output is returned in fp32: the result is within the bf16
    tolerance of fp32 attention, not fp32-exact."""
    dev = _require_cuda(q, k, v)
    if past_dev is not None:
        if unmasked:
            raise ValueError("a device-side prefix length needs the tree or causal mask")
        if past_dev.dtype != torch.int64 or not past_dev.is_cuda or past_dev.numel() != 1:
            raise ValueError("past_dev must be a device i64 [1]")
    if q.dtype == torch.float32 and k.dtype == torch.float32 and v.dtype == torch.float32:
        if past_dev is not None:
            raise TypeError("a device-side prefix length takes bf16 q / k / v")
        res = tree_attention(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16),
                             anc_bits, past_length, scale=scale, causal=causal,
                             kv_splits=kv_splits, status=status, unmasked=unmasked)
        if out is None:
            return res.float()
        out.copy_(res)
        return out
    n, hq, qns, qhs = _q_view(q)
    hkv, s, khs, kss = _kv_view(k)
    _, _, vhs, vss = _kv_view(v)
    if (khs, kss) != (vhs, vss):
        raise ValueError("k and v must share strides")
    d = q.shape[-1]
    if s != past_length + n:
        raise ValueError(f"key length {s} != past_length + nodes ({past_length} + {n})")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise TypeError("tree attention takes bf16 (or all-fp32) q / k / v")
    if out is None:
        out = torch.empty((n, hq, d), dtype=torch.bfloat16, device=dev)
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    lib = _lib.load()
    ws_bytes = lib.ddt_tree_attn_workspace_bytes(n, hq, d, kv_splits)
    ws = WORKSPACES.get(dev, "tree_attn", ws_bytes)
    if status is None:
        status = attention_status(dev)
    mode = _mask_mode(causal, unmasked)
    if mode == DDT_MASK_TREE and anc_bits is None:
        raise ValueError("tree mode needs ancestor bitmasks")
    words = anc_bits.shape[1] if anc_bits is not None else 0
    stream = _stream(dev)
    if STATS.time_attention:
        # external events are recorded as graph nodes when captured, so they also time
        # the launch inside a replayed CUDA graph
        ev = (torch.cuda.Event(enable_timing=True, external=True),
              torch.cuda.Event(enable_timing=True, external=True))
        ev[0].record()
    if past_dev is not None:
        rc = lib.ddt_tree_attn_device_past(
            q.data_ptr(), qns, qhs, k.data_ptr(), v.data_ptr(), khs, kss, out.data_ptr(),
            out.stride(0), out.stride(1), n, past_length, past_dev.data_ptr(), hq, hkv, d,
            anc_bits.data_ptr() if anc_bits is not None else None, words, mode, float(scale),
            kv_splits, ws.data_ptr(), ws.numel(), status.data_ptr(), stream)
        check(rc, "ddt_tree_attn_device_past")
    else:
        rc = lib.ddt_tree_attn(
            q.data_ptr(), qns, qhs, k.data_ptr(), v.data_ptr(), khs, kss, out.data_ptr(),
            out.stride(0), out.stride(1), n, past_length, hq, hkv, d,
            anc_bits.data_ptr() if anc_bits is not None else None, words, mode, float(scale),
            kv_splits, ws.data_ptr(), ws.numel(), status.data_ptr(), stream)
        check(rc, "ddt_tree_attn")
    if STATS.time_attention:
        ev[1].record()
        STATS.attn_events.append(ev)
    STATS.launches += 1 + (1 if attn_splits(n, hq, hkv, past_length, kv_splits) > 1 else 0)
    return out


def attn_splits(n_nodes: int, q_heads: int, kv_heads: int, past_length: int,
                kv_splits: int = 0) -> int:
    """The key-range split count ddt_tree_attn uses (asked of the library, which picks it)."""
    if kv_splits > 0:
        return kv_splits
    return int(_lib.load().ddt_tree_attn_partial_splits(n_nodes, past_length + n_nodes, q_heads,
                                                        kv_heads))


def tree_attention_partial(q, k_shard, v_shard, key_begin: int, key_end: int, anc_bits,
                           past_length: int, scale: float | None = None, causal: bool = False,
                           out=None, status=None, kv_splits: int = 0):
    """Partials (O unnormalised fp32 [S, N*Hq, D], m [S, N*Hq], l [S, N*Hq]) over global keys
    [key_begin, key_end), whose K/V rows are k_shard / v_shard ([Hkv, key_end - key_begin,
    D]); S = kv_splits in-GPU key splits (0 picks enough to fill the GPU)."""
    dev = _require_cuda(q, k_shard, v_shard)
    n, hq, qns, qhs = _q_view(q)
    hkv, s_local, khs, kss = _kv_view(k_shard)
    d = q.shape[-1]
    if s_local < key_end - key_begin:
        raise ValueError("shard shorter than its key range")
    lib = _lib.load()
    if kv_splits <= 0:
        kv_splits = int(lib.ddt_tree_attn_partial_splits(n, key_end - key_begin, hq, hkv))
    if out is None:
        out = (torch.empty((kv_splits, n * hq, d), dtype=torch.float32, device=dev),
               torch.empty((kv_splits, n * hq), dtype=torch.float32, device=dev),
               torch.empty((kv_splits, n * hq), dtype=torch.float32, device=dev))
    o, m, l = out
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if status is None:
        status = attention_status(dev)
    words = anc_bits.shape[1] if anc_bits is not None else 0
    rc = lib.ddt_tree_attn_partial(
        q.data_ptr(), qns, qhs, k_shard.data_ptr(), v_shard.data_ptr(), khs, kss, key_begin,
        key_end, o.data_ptr(), m.data_ptr(), l.data_ptr(), n, past_length, hq, hkv, d,
        anc_bits.data_ptr() if anc_bits is not None else None, words,
        DDT_MASK_CAUSAL if causal else DDT_MASK_TREE, float(scale), kv_splits, status.data_ptr(),
        _stream(dev))
    check(rc, "ddt_tree_attn_partial")
    STATS.launches += 1
    return o, m, l


def tree_attention_partial_merged(q, k_shard, v_shard, key_begin: int, key_end: int, anc_bits,
                                  past_length: int, scale: float | None = None,
                                  causal: bool = False, out=None, status=None):
    """One partial per row over global keys [key_begin, key_end): (O unnormalised fp32
    [N*Hq, D], m [N*Hq], l [N*Hq]).  The shard's key tiles are spread over all SMs and merged
    in-GPU (ddt_tree_attn_partial_merged), so a cross-GPU exchange moves one partial per
    row and rank."""
    dev = _require_cuda(q, k_shard, v_shard)
    n, hq, qns, qhs = _q_view(q)
    hkv, s_local, khs, kss = _kv_view(k_shard)
    d = q.shape[-1]
    if s_local < key_end - key_begin:
        raise ValueError("shard shorter than its key range")
    lib = _lib.load()
    if out is None:
        out = (torch.empty((n * hq, d), dtype=torch.float32, device=dev),
               torch.empty((n * hq,), dtype=torch.float32, device=dev),
               torch.empty((n * hq,), dtype=torch.float32, device=dev))
    o, m, l = out
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if status is None:
        status = attention_status(dev)
    ws_bytes = lib.ddt_tree_attn_partial_merged_workspace_bytes(n, hq, d)
    ws = WORKSPACES.get(dev, "attn_partial_merged", ws_bytes)
    words = anc_bits.shape[1] if anc_bits is not None else 0
    rc = lib.ddt_tree_attn_partial_merged(
        q.data_ptr(), qns, qhs, k_shard.data_ptr(), v_shard.data_ptr(), khs, kss, key_begin,
        key_end, o.data_ptr(), m.data_ptr(), l.data_ptr(), n, past_length, hq, hkv, d,
        anc_bits.data_ptr() if anc_bits is not None else None, words,
        DDT_MASK_CAUSAL if causal else DDT_MASK_TREE, float(scale), ws.data_ptr(), ws.numel(),
        status.data_ptr(), _stream(dev))
    check(rc, "ddt_tree_attn_partial_merged")
    STATS.launches += 2
    return o, m, l


def tree_attention_wait_check(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                              anc_bits: torch.Tensor, past_length: int, timeout_ns: int,
                              status: torch.Tensor) -> torch.Tensor:
    """ddt_tree_attn_wait_check: one attention launch whose producer withholds every load,
    so each wait of the kernel runs out after timeout_ns; returns the output buffer (zeros
    where the kernel reached its epilogue).  The caller reads `status` afterwards."""
    dev = _require_cuda(q, k, v, anc_bits, status)
    n, hq, d = q.shape
    hkv = k.shape[0]
    for t in (q, k, v):
        if not t.is_contiguous() or t.dtype != torch.bfloat16:
            raise ValueError("contiguous bf16 q / k / v expected")
    out = torch.zeros_like(q)
    check(_lib.load().ddt_tree_attn_wait_check(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), n, past_length, hq, hkv,
        anc_bits.data_ptr(), anc_bits.shape[1], int(timeout_ns), status.data_ptr(),
        _stream(dev)), "ddt_tree_attn_wait_check")
    STATS.launches += 1
    return out


def attn_merge(o_parts: torch.Tensor, m_parts: torch.Tensor, l_parts: torch.Tensor, n_nodes: int,
               q_heads: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Merges [P, rows, D] / [P, rows] partials into bf16 [n_nodes, q_heads, D]."""
    dev = _require_cuda(o_parts, m_parts, l_parts)
    d = o_parts.shape[-1]
    if out is None:
        out = torch.empty((n_nodes, q_heads, d), dtype=torch.bfloat16, device=dev)
    check(_lib.load().ddt_attn_merge(o_parts.data_ptr(), m_parts.data_ptr(), l_parts.data_ptr(),
                                     o_parts.shape[0], n_nodes, q_heads, d, out.data_ptr(),
                                     out.stride(0), out.stride(1), _stream(dev)), "ddt_attn_merge")
    STATS.launches += 1
    return out


def mask_to_bits(mask_block: torch.Tensor, words: int | None = None) -> torch.Tensor:
    """[N, N] additive mask block (0 = visible) -> i32 [N, words] ancestor bitmasks."""
    dev = _require_cuda(mask_block)
    n = mask_block.shape[0]
    words = anc_words_for(n) if words is None else words
    if mask_block.stride(1) != 1:
        mask_block = mask_block.contiguous()
    bits = torch.empty((n, words), dtype=torch.int32, device=dev)
    check(_lib.load().ddt_mask_to_bits(mask_block.data_ptr(), _dtype_code(mask_block), n,
                                       mask_block.stride(0), bits.data_ptr(), words, _stream(dev)),
          "ddt_mask_to_bits")
    STATS.launches += 1
    return bits
