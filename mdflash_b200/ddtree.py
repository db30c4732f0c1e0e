"""Drop-in replacements for the DDTree tree utilities (ddtree.py of the DDTree research
code), same names, arguments, return types and error behaviour, running on the B200
kernels of ``libddtree_b200.so``:

  build_ddtree_tree        ddtree.py:84-166
  build_sampled_candidate_tree  ddtree.py:169-224
  compile_ddtree_tree      ddtree.py:227-267
  follow_verified_tree     ddtree.py:270-281
  compact_dynamic_cache    ddtree.py:303-335
  load_cpp_compact_module  ddtree.py:22-74 (its compact_tail_inplace, :31-58)
  maybe_enable_cpp_compact ddtree.py:77-81

The reference returns host objects (CPU tensors, lists, dicts) from the tree build, so
these functions copy the finished tree back once; they also keep the device-resident
tree (ancestor bitmasks, parents, node tokens) in a per-thread context, which
``compile_ddtree_tree`` hands to the ``ddtree_tree`` attention plug-in and which
``follow_verified_tree`` walks on the device.  Code that wants no host round trip at all
uses :class:`mdflash_b200.verifier.TreeVerifier`.

All inputs must be CUDA tensors: there is no CPU path.
"""
from __future__ import annotations

import time
from types import SimpleNamespace

import numpy as np
import torch

from . import attention as A
from . import kernels as K

DDTREE_STAGE_ORDER = ("draft", "tree_build", "tree_compile", "verify", "commit")
DDTREE_TREE_BUILD_STAGE_ORDER = ("tree_build_copy", "tree_build_heap", "tree_build_visibility")


class _LastTree:
    tree: K.DeviceTree | None = None
    n_nodes: int = 0


_LAST = _LastTree()


def _empty_stage_times(names):
    return {n: 0.0 for n in names}


def _require_cuda_tensor(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor: mdflash_b200 runs on the GPU only")


def unpack_visibility(anc_bits: np.ndarray, n: int) -> np.ndarray:
    """i32/u32 [n, words] ancestor bitmasks -> bool [n, n] visibility."""
    b = np.ascontiguousarray(anc_bits[:n]).view(np.uint8)
    return np.unpackbits(b, axis=-1, bitorder="little", count=n).astype(bool)


def build_ddtree_tree(draft_logits: torch.Tensor, budget: int):
    """ddtree.py:84-166.  Returns (node_token_ids i64 CPU [B'], node_depths i64 CPU [B'],
    parents list[int] (len B'+1, parents[0] = -1), child_maps list[dict[int, int]],
    visibility bool CPU [B'+1, B'+1], subtimes dict)."""
    subtimes = _empty_stage_times(DDTREE_TREE_BUILD_STAGE_ORDER)
    if budget <= 0 or draft_logits.shape[0] == 0:
        visibility = torch.zeros((1, 1), dtype=torch.bool)
        visibility[0, 0] = True
        _LAST.tree, _LAST.n_nodes = None, 1
        return (torch.empty(0, dtype=torch.long), torch.empty(0, dtype=torch.long), [-1], [dict()],
                visibility, subtimes)
    _require_cuda_tensor(draft_logits, "draft_logits")
    t0 = time.perf_counter()
    tree = K.topk_tree(draft_logits, budget)
    n = tree.n_nodes
    cnt = n - 1
    # one device->host copy of the finished tree
    host = torch.cat([tree.node_token_ids[:cnt], tree.node_depths[:cnt],
                      tree.parents[:n].to(torch.int64),
                      tree.anc_bits[:n].reshape(-1).to(torch.int64)]).cpu()
    t1 = time.perf_counter()
    node_ids = host[:cnt].clone()
    depths = host[cnt:2 * cnt].clone()
    parents_np = host[2 * cnt:2 * cnt + n].numpy()
    bits = host[2 * cnt + n:].numpy().astype(np.uint32).reshape(n, tree.anc_words)
    t2 = time.perf_counter()
    vis = torch.from_numpy(unpack_visibility(bits, n))
    parents = parents_np.astype(np.int64).tolist()
    child_maps: list[dict[int, int]] = [dict() for _ in range(n)]
    ids_list = node_ids.tolist()
    for i in range(1, n):
        child_maps[parents[i]][ids_list[i - 1]] = i
    t3 = time.perf_counter()
    subtimes.update(tree_build_copy=t1 - t0, tree_build_heap=t2 - t1, tree_build_visibility=t3 - t2)
    _LAST.tree, _LAST.n_nodes = tree, n
    return node_ids, depths, parents, child_maps, vis, subtimes


def _host_tree(tree: K.DeviceTree, n: int):
    """One device->host copy of a built tree: (node_ids, depths, parents list, child_maps,
    visibility) in the reference's types."""
    cnt = n - 1
    host = torch.cat([tree.node_token_ids[:cnt], tree.node_depths[:cnt],
                      tree.parents[:n].to(torch.int64),
                      tree.anc_bits[:n].reshape(-1).to(torch.int64)]).cpu()
    node_ids = host[:cnt].clone()
    depths = host[cnt:2 * cnt].clone()
    parents_np = host[2 * cnt:2 * cnt + n].numpy()
    bits = host[2 * cnt + n:].numpy().astype(np.uint32).reshape(n, tree.anc_words)
    vis = torch.from_numpy(unpack_visibility(bits, n))
    parents = parents_np.astype(np.int64).tolist()
    child_maps: list[dict[int, int]] = [dict() for _ in range(n)]
    ids_list = node_ids.tolist()
    for i in range(1, n):
        child_maps[parents[i]][ids_list[i - 1]] = i
    return node_ids, depths, parents, child_maps, vis


def build_sampled_candidate_tree(candidate_token_ids: torch.Tensor, budget: int):
    """ddtree.py:169-224: the trie of the sampled chains (i64 [num_chains, depths], chain
    order, at most `budget` nodes), built on the device by ddt_chain_tree.  Returns
    (node_token_ids i64 CPU, node_depths i64 CPU, parents list, child_maps list[dict],
    visibility bool CPU [N, N]) like the reference, and registers the device tree for
    compile_ddtree_tree / the attention plug-in / follow_verified_tree."""
    if (budget <= 0 or candidate_token_ids.dim() != 2 or candidate_token_ids.shape[0] == 0
            or candidate_token_ids.shape[1] == 0):
        visibility = torch.zeros((1, 1), dtype=torch.bool)
        visibility[0, 0] = True
        _LAST.tree, _LAST.n_nodes = None, 1
        return (torch.empty(0, dtype=torch.long), torch.empty(0, dtype=torch.long), [-1], [dict()],
                visibility)
    _require_cuda_tensor(candidate_token_ids, "candidate_token_ids")
    tree = K.chain_tree(candidate_token_ids, budget)
    n = 1 + int(tree.node_count.item())
    tree.n_nodes = n
    node_ids, depths, parents, child_maps, vis = _host_tree(tree, n)
    _LAST.tree, _LAST.n_nodes = tree, n
    return node_ids, depths, parents, child_maps, vis


def compile_ddtree_tree(root_token_id, start: int, node_token_ids: torch.Tensor,
                        node_depths: torch.Tensor, visibility_cpu: torch.Tensor, past_length: int,
                        dtype: torch.dtype, device, verify_input_ids_buffer: torch.Tensor,
                        verify_position_ids_buffer: torch.Tensor,
                        attention_mask_buffer: torch.Tensor, tree_visibility_buffer: torch.Tensor,
                        previous_tree_start: int, previous_tree_length: int):
    """ddtree.py:227-267: fills the verify ids / positions / visibility / additive-mask
    buffers exactly like the reference and returns (ids, pos, mask, past_length,
    current_length).  When the tree is the one ``build_ddtree_tree`` just built, the
    ids, positions and visibility come from the device-resident tree (no host->device
    copy), and the tree is registered for the ``ddtree_tree`` attention plug-in."""
    n = 1 + int(node_token_ids.numel())
    _require_cuda_tensor(verify_input_ids_buffer, "verify_input_ids_buffer")
    if previous_tree_length > 0:
        attention_mask_buffer[0, 0, :previous_tree_length,
                              previous_tree_start:previous_tree_start + previous_tree_length] = 0
    ids = verify_input_ids_buffer[:, :n]
    pos = verify_position_ids_buffer[:, :n]
    vis = tree_visibility_buffer[:n, :n]
    tree = _LAST.tree if (_LAST.tree is not None and _LAST.n_nodes == n) else None
    if tree is not None:
        ids[0, 1:n].copy_(tree.node_token_ids[:n - 1])
        pos[0, 1:n].copy_(tree.node_depths[:n - 1])
        bits = tree.anc_bits[:n]
        words = torch.arange(n, device=bits.device)
        dev_vis = ((bits[:, words // 32] >> (words % 32)) & 1).bool()
        vis.copy_(dev_vis)
    else:
        if n > 1:
            ids[0, 1:n].copy_(node_token_ids, non_blocking=False)
            pos[0, 1:n].copy_(node_depths, non_blocking=False)
        vis.copy_(visibility_cpu, non_blocking=False)
    ids[0, 0] = root_token_id
    pos[0, 0] = 0
    pos[0, :n].add_(start)
    block = attention_mask_buffer[0, 0, :n, past_length:past_length + n]
    block.fill_(torch.finfo(dtype).min)
    block.masked_fill_(vis, 0)
    mask = attention_mask_buffer[:, :, :n, :past_length + n]
    if tree is not None:
        A.set_tree_context(tree, past_length, n)
    else:
        A.clear_tree_context()
    return ids, pos, mask, past_length, n


def follow_verified_tree(child_maps: list[dict[int, int]], posterior: torch.Tensor):
    """ddtree.py:270-281: greedy walk from the root; returns (accepted_indices, next_token).
    The walk runs on the device (ddt_accept_compact without cache tensors): over the tree
    registered by ``build_ddtree_tree`` when ``child_maps`` describes that tree, otherwise over
    the tree ``child_maps`` describes, copied to the device first.  Raises DDTreeError
    (DDT_ERR_TIMEOUT) if the verify attention reported a bounded-wait timeout."""
    _require_cuda_tensor(posterior, "posterior")
    n = len(child_maps)
    post = posterior.reshape(-1)
    tree = _LAST.tree
    status = K.attention_status(post.device)
    if tree is not None and _LAST.n_nodes == n and post.numel() >= n:
        empty = _EmptyKv.get(post.device)
        acc, cnt, nxt = K.accept_compact(post[:n], tree, empty, 0, n_nodes=n)
        host = torch.cat([status.to(torch.int64), cnt.to(torch.int64), nxt, acc]).cpu().tolist()
        if host[0] != 0:  # the verify attention gave up a bounded wait: the posterior is void
            K.check_status(status, "tree attention of the verify forward")
        c = host[1]
        return host[3:3 + c], int(host[2])
    # a tree this thread did not just build: its topology goes to the device and the same
    # walk kernel runs over it
    foreign = _tree_from_child_maps(child_maps, post.device)
    if post.numel() < n:
        raise ValueError("posterior shorter than the tree")
    acc, cnt, nxt = K.accept_compact(post[:n], foreign, _EmptyKv.get(post.device), 0, n_nodes=n)
    host = torch.cat([status.to(torch.int64), cnt.to(torch.int64), nxt, acc]).cpu().tolist()
    if host[0] != 0:
        K.check_status(status, "tree attention of the verify forward")
    c = host[1]
    return host[3:3 + c], int(host[2])


def _tree_from_child_maps(child_maps: list[dict[int, int]], device) -> SimpleNamespace:
    """Parents (i32 [n]) and node tokens (i64 [n - 1]) of the tree child_maps describes
    (child_maps[p][token] = child, node i >= 1 carries token node_token_ids[i - 1])."""
    n = len(child_maps)
    parents = np.full(n, -1, np.int32)
    tokens = np.zeros(max(n - 1, 1), np.int64)
    for p, m in enumerate(child_maps):
        for tok, c in m.items():
            if not 0 < c < n or parents[c] != -1:
                raise ValueError("child_maps does not describe a tree over nodes 0..n-1")
            parents[c] = p
            tokens[c - 1] = int(tok)
    if n > 1 and (parents[1:] < 0).any():
        raise ValueError("child_maps leaves a node without a parent")
    depth = np.zeros(n, np.int64)
    for c in range(1, n):  # a walk accepts at most DDT_MAX_DEPTH nodes below the root
        d, j = 0, c
        while j > 0 and d <= n:
            j = int(parents[j])
            d += 1
        if d > n:
            raise ValueError("child_maps contains a cycle")
        depth[c] = d
    if n > 1 and depth.max() > K._lib.DDT_MAX_DEPTH:
        raise ValueError(f"tree deeper than {K._lib.DDT_MAX_DEPTH} levels")
    return SimpleNamespace(parents=torch.from_numpy(parents).to(device),
                           node_token_ids=torch.from_numpy(tokens).to(device), n_nodes=n)


class _EmptyKv:
    """A zero-tensor KV table: lets the fused kernel run the walk alone."""
    _cache: dict = {}

    @classmethod
    def get(cls, device):
        t = cls._cache.get(device)
        if t is None:
            dummy = torch.zeros((1, 1, 8), dtype=torch.bfloat16, device=device)
            t = K.KvTable([dummy])
            t.n = 0
            t.seq = 1 << 30
            cls._cache[device] = t
        return t


def _cache_tensors(past_key_values):
    if hasattr(past_key_values, "key_cache") and hasattr(past_key_values, "value_cache"):
        ks, vs = past_key_values.key_cache, past_key_values.value_cache
        return [t for kv in zip(ks, vs) for t in kv]
    if hasattr(past_key_values, "layers"):
        ts = []
        for layer in past_key_values.layers:
            if not hasattr(layer, "keys") or layer.keys is None or layer.keys.numel() == 0:
                continue
            ts += [layer.keys, layer.values]
        return ts
    raise RuntimeError("Unsupported DynamicCache layout for DDTree cache compaction.")


def compact_dynamic_cache(past_key_values, past_length: int, keep_current_indices: list[int]) -> None:
    """ddtree.py:303-335: rows past_length + keep[j] move to past_length + j in every
    layer's K and V (one kernel launch for the whole cache), then crop to
    past_length + len(keep)."""
    if len(keep_current_indices) == 0:
        past_key_values.crop(past_length)
        return
    tensors = _cache_tensors(past_key_values)
    keep = [int(i) for i in keep_current_indices]
    by_dev: dict = {}
    for t in tensors:
        by_dev.setdefault(t.device, []).append(t)
    for dev, ts in by_dev.items():
        _require_cuda_tensor(ts[0], "cache tensors")
        cur = ts[0].shape[-2] - past_length
        if cur <= 0 or len(keep) == cur:
            continue  # reference no-op cases (ddtree.py:285-291)
        if len(keep) > cur:
            raise RuntimeError("keep_count exceeds appended window length")
        table = getattr(past_key_values, "kv_table", None)
        kv = table() if table is not None else K.KvTable(ts)
        K.compact_kv(keep, kv, past_length)
    past_key_values.crop(past_length + len(keep))


class _CompactModule:
    """Mirror of the reference's inline C++ extension (ddtree.py:31-58)."""

    @staticmethod
    def compact_tail_inplace(cache_tensor: torch.Tensor, past_length: int,
                             keep_current_indices: torch.Tensor) -> torch.Tensor:
        if cache_tensor.dim() < 2:
            raise RuntimeError("cache_tensor must have rank >= 2")
        if keep_current_indices.dim() != 1:
            raise RuntimeError("keep_current_indices must be a 1D tensor")
        if keep_current_indices.dtype != torch.long:
            raise RuntimeError("keep_current_indices must have dtype torch.long")
        if cache_tensor.device != keep_current_indices.device:
            raise RuntimeError("cache_tensor and keep_current_indices must be on the same device")
        seq = cache_tensor.shape[-2]
        if past_length < 0:
            raise RuntimeError("past_length must be non-negative")
        if past_length > seq:
            raise RuntimeError("past_length exceeds cache sequence length")
        cur = seq - past_length
        if cur <= 0:
            return cache_tensor
        keep_count = keep_current_indices.numel()
        if keep_count > cur:
            raise RuntimeError("keep_count exceeds appended window length")
        if keep_count == 0 or keep_count == cur:
            return cache_tensor
        _require_cuda_tensor(cache_tensor, "cache_tensor")
        t = cache_tensor.reshape(-1, seq, cache_tensor.shape[-1])
        if t.data_ptr() != cache_tensor.data_ptr():
            raise RuntimeError("cache_tensor must be viewable as [heads, seq, head_dim]")
        K.compact_kv(keep_current_indices, K.KvTable([t]), past_length)
        return cache_tensor


_CPP_COMPACT_ENABLED = True


def load_cpp_compact_module():
    """The reference builds an inline C++ extension here; the B200 compaction kernel is
    part of libddtree_b200.so, so this returns its Python face."""
    from . import _lib
    _lib.load()
    return _CompactModule()


def maybe_enable_cpp_compact(enabled: bool) -> None:
    global _CPP_COMPACT_ENABLED
    _CPP_COMPACT_ENABLED = enabled
    if enabled:
        load_cpp_compact_module()


def empty_stage_times(stage_names):
    return _empty_stage_times(stage_names)


def result_namespace(**kw) -> SimpleNamespace:
    return SimpleNamespace(**kw)
