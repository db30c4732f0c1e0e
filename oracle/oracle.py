"""Python side of the CPU oracle (test infrastructure only; see oracle/__init__.py).

Integer and topology work runs in the C restatement ``ddtree_oracle.c`` (loaded with
ctypes); byte moves are numpy; the floating-point attention check is torch fp32 on the
CPU, the same ``scaled_dot_product_attention`` call the reference makes.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import time
from dataclasses import dataclass

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_NAME = "libddtree_oracle.so"
_lib = None


def library_path() -> str:
    return os.path.join(_HERE, _LIB_NAME)


def build_library(force: bool = False) -> str:
    path = library_path()
    src = os.path.join(_HERE, "ddtree_oracle.c")
    if force or not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return path


def _load():
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not os.path.exists(path):
        build_library()
    lib = ctypes.CDLL(path)
    P = ctypes.c_void_p
    I = ctypes.c_int64
    lib.orc_logz_topk.argtypes = [P, I, I, I, P, P, P]
    lib.orc_build_tree.argtypes = [P, P, I, I, I, P, P, P, P]
    lib.orc_visibility.argtypes = [P, I, P]
    lib.orc_ancestor_bits.argtypes = [P, I, I, P]
    lib.orc_argmax.argtypes = [P, I, I, P]
    lib.orc_follow.argtypes = [P, P, I, P, P, P, P]
    for f in (lib.orc_logz_topk, lib.orc_build_tree, lib.orc_visibility, lib.orc_ancestor_bits,
              lib.orc_argmax, lib.orc_follow):
        f.restype = ctypes.c_int
    _lib = lib
    return lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed with code {rc}")


def _as_f32_rows(draft_logits) -> np.ndarray:
    if isinstance(draft_logits, torch.Tensor):
        return np.ascontiguousarray(draft_logits.detach().to("cpu", torch.float32).numpy())
    return np.ascontiguousarray(np.asarray(draft_logits, dtype=np.float32))


def logz_topk(draft_logits, k: int):
    """ddtree.py:106-110 with the canonical tie rule.  Returns (top_lp f32 [L,k],
    top_ids i64 [L,k], logz f32 [L])."""
    x = _as_f32_rows(draft_logits)
    L, V = x.shape
    top_lp = np.empty((L, k), np.float32)
    top_ids = np.empty((L, k), np.int64)
    logz = np.empty((L,), np.float32)
    _check(_load().orc_logz_topk(_ptr(x), L, V, k, _ptr(top_lp), _ptr(top_ids), _ptr(logz)),
           "logz_topk")
    return top_lp, top_ids, logz


def build_tree(top_lp: np.ndarray, top_ids: np.ndarray, budget: int):
    """ddtree.py:116-147.  Returns (node_ids i64 [n], depths i64 [n], parents i32 [n+1])."""
    top_lp = np.ascontiguousarray(top_lp, np.float32)
    top_ids = np.ascontiguousarray(top_ids, np.int64)
    L, k = top_lp.shape
    nb = max(budget, 1)
    node_ids = np.zeros(nb, np.int64)
    depths = np.zeros(nb, np.int64)
    parents = np.zeros(nb + 1, np.int32)
    count = np.zeros(1, np.int64)
    _check(_load().orc_build_tree(_ptr(top_lp), _ptr(top_ids), L, k, budget, _ptr(node_ids),
                                  _ptr(depths), _ptr(parents), _ptr(count)), "build_tree")
    n = int(count[0])
    return node_ids[:n].copy(), depths[:n].copy(), parents[: n + 1].copy()


def visibility(parents: np.ndarray) -> np.ndarray:
    parents = np.ascontiguousarray(parents, np.int32)
    n = parents.shape[0]
    vis = np.zeros((n, n), np.uint8)
    _check(_load().orc_visibility(_ptr(parents), n, _ptr(vis)), "visibility")
    return vis.astype(bool)


def ancestor_bits(parents: np.ndarray, words: int | None = None) -> np.ndarray:
    parents = np.ascontiguousarray(parents, np.int32)
    n = parents.shape[0]
    words = (n + 31) // 32 if words is None else words
    bits = np.zeros((n, words), np.uint32)
    _check(_load().orc_ancestor_bits(_ptr(parents), n, words, _ptr(bits)), "ancestor_bits")
    return bits


@dataclass
class OracleTree:
    node_ids: np.ndarray
    depths: np.ndarray
    parents: np.ndarray
    top_lp: np.ndarray
    top_ids: np.ndarray
    logz: np.ndarray


def build_ddtree_tree(draft_logits: torch.Tensor, budget: int):
    """Restatement of ddtree.py:84-166 with the same return types:
    (node_token_ids i64 CPU, node_depths i64 CPU, parents list, child_maps list[dict],
    visibility bool [N,N] CPU, subtimes dict)."""
    subtimes = {"tree_build_copy": 0.0, "tree_build_heap": 0.0, "tree_build_visibility": 0.0}
    if budget <= 0 or draft_logits.shape[0] == 0:
        vis = torch.zeros((1, 1), dtype=torch.bool)
        vis[0, 0] = True
        return (torch.empty(0, dtype=torch.long), torch.empty(0, dtype=torch.long), [-1],
                [dict()], vis, subtimes)
    k = min(budget, draft_logits.shape[-1])
    t0 = time.perf_counter()
    top_lp, top_ids, _ = logz_topk(draft_logits, k)
    t1 = time.perf_counter()
    node_ids, depths, parents = build_tree(top_lp, top_ids, budget)
    t2 = time.perf_counter()
    vis = visibility(parents)
    t3 = time.perf_counter()
    subtimes.update(tree_build_copy=t1 - t0, tree_build_heap=t2 - t1, tree_build_visibility=t3 - t2)
    child_maps: list[dict[int, int]] = [dict() for _ in range(parents.shape[0])]
    for i in range(1, parents.shape[0]):
        child_maps[int(parents[i])][int(node_ids[i - 1])] = i
    return (torch.from_numpy(node_ids), torch.from_numpy(depths), parents.tolist(), child_maps,
            torch.from_numpy(vis), subtimes)


def build_sampled_candidate_tree(candidate_token_ids, budget: int):
    """Restatement of ddtree.py:169-224 (the trie of sampled chains, in chain order, stopping
    at the first new node past the budget) with the same return types: (node_token_ids i64
    CPU, node_depths i64 CPU, parents list, child_maps list[dict], visibility bool [N, N])."""
    chains = np.asarray(candidate_token_ids, np.int64)
    if budget <= 0 or chains.ndim != 2 or chains.shape[0] == 0 or chains.shape[1] == 0:
        vis = torch.zeros((1, 1), dtype=torch.bool)
        vis[0, 0] = True
        return torch.empty(0, dtype=torch.long), torch.empty(0, dtype=torch.long), [-1], [dict()], vis
    parents = [-1]
    child_maps: list[dict[int, int]] = [dict()]
    tokens: list[int] = []
    depths: list[int] = []
    full = False
    for chain in chains.tolist():
        cur = 0
        for depth, tok in enumerate(chain, start=1):
            nxt = child_maps[cur].get(tok)
            if nxt is None:
                if len(tokens) >= budget:
                    full = True
                    break
                nxt = len(parents)
                parents.append(cur)
                child_maps.append(dict())
                child_maps[cur][tok] = nxt
                tokens.append(tok)
                depths.append(depth)
            cur = nxt
        if full:
            break
    par = np.asarray(parents, np.int32)
    return (torch.tensor(tokens, dtype=torch.long), torch.tensor(depths, dtype=torch.long), parents,
            child_maps, torch.from_numpy(visibility(par)))


def compile_ddtree_tree(root_token_id, start, node_token_ids, node_depths, visibility_cpu,
                        past_length, dtype, device, verify_input_ids_buffer,
                        verify_position_ids_buffer, attention_mask_buffer, tree_visibility_buffer,
                        previous_tree_start, previous_tree_length):
    """Restatement of ddtree.py:227-267 (same buffers, same return tuple)."""
    n = 1 + int(node_token_ids.numel())
    if previous_tree_length > 0:
        attention_mask_buffer[0, 0, :previous_tree_length,
                              previous_tree_start:previous_tree_start + previous_tree_length] = 0
    ids = verify_input_ids_buffer[:, :n]
    ids[0, 0] = root_token_id
    pos = verify_position_ids_buffer[:, :n]
    pos[0, 0] = start
    if n > 1:
        ids[0, 1:n].copy_(node_token_ids)
        pos[0, 1:n].copy_(node_depths)
        pos[0, 1:n].add_(start)
    vis = tree_visibility_buffer[:n, :n]
    vis.copy_(visibility_cpu)
    block = attention_mask_buffer[0, 0, :n, past_length:past_length + n]
    block.fill_(torch.finfo(dtype).min)
    block.masked_fill_(vis, 0)
    mask = attention_mask_buffer[:, :, :n, :past_length + n]
    return ids, pos, mask, past_length, n


def argmax(logits) -> np.ndarray:
    """model/utils.py:28-30 at temperature 0: row argmax, lowest index on ties."""
    x = _as_f32_rows(logits.reshape(-1, logits.shape[-1]) if isinstance(logits, torch.Tensor)
                     else np.asarray(logits).reshape(-1, np.asarray(logits).shape[-1]))
    out = np.empty((x.shape[0],), np.int64)
    _check(_load().orc_argmax(_ptr(x), x.shape[0], x.shape[1], _ptr(out)), "argmax")
    return out


def follow_verified_tree(child_maps_or_tree, posterior):
    """ddtree.py:270-281.  Accepts the reference child_maps list, or a (parents,
    node_ids) pair, and a posterior of shape [1, N] or [N]."""
    post = np.ascontiguousarray(
        (posterior.detach().cpu().numpy() if isinstance(posterior, torch.Tensor)
         else np.asarray(posterior)).reshape(-1).astype(np.int64))
    if isinstance(child_maps_or_tree, list):
        cm = child_maps_or_tree
        accepted = [0]
        cur = 0
        tok = int(post[cur])
        while tok in cm[cur]:
            cur = cm[cur][tok]
            accepted.append(cur)
            tok = int(post[cur])
        return accepted, tok
    parents, node_ids = child_maps_or_tree
    parents = np.ascontiguousarray(parents, np.int32)
    node_ids = np.ascontiguousarray(node_ids, np.int64)
    n = parents.shape[0]
    acc = np.zeros(n + 1, np.int64)
    cnt = np.zeros(1, np.int64)
    nxt = np.zeros(1, np.int64)
    _check(_load().orc_follow(_ptr(parents), _ptr(node_ids), n, _ptr(post), _ptr(acc), _ptr(cnt),
                              _ptr(nxt)), "follow")
    return acc[: int(cnt[0])].tolist(), int(nxt[0])


def compact_rows(cache: np.ndarray, past_length: int, keep) -> np.ndarray:
    """ddtree.py:284-300 on one [..., S, D] array: rows past_length + keep[j] move to
    past_length + j (numpy fancy indexing reads before it writes), then the result is
    cropped to past_length + len(keep).  Returns the cropped view."""
    keep = np.asarray(keep, np.int64)
    cur = cache.shape[-2] - past_length
    if cur <= 0:
        return cache
    if keep.size == 0:
        return cache[..., :past_length, :]
    if keep.size != cur:
        cache[..., past_length:past_length + keep.size, :] = cache[..., past_length + keep, :]
    return cache[..., :past_length + keep.size, :]


def compact_dynamic_cache(layers, past_length: int, keep_current_indices: list[int]):
    """ddtree.py:303-335 over a list of (keys, values) arrays; returns the cropped list."""
    return [(compact_rows(k, past_length, keep_current_indices),
             compact_rows(v, past_length, keep_current_indices)) for k, v in layers]


def tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, vis: np.ndarray | None,
                   past_length: int, scale: float | None = None, causal: bool = False):
    """softmax(Q K^T * scale + mask) V in fp32 on the CPU, the way the reference's verify
    forward reaches torch SDPA (transformers sdpa_attention.py:92-101, enable_gqa) with the
    additive mask of ddtree.py:262-264 (0 where visible, finfo.min elsewhere).

    q: [Hq, N, D]; k, v: [Hkv, S, D] with S = past_length + N; vis: bool [N, N] or None
    (with causal=True: node i sees keys < past_length + i + 1).  Returns [N, Hq, D] fp32."""
    qf = q.float().unsqueeze(0)
    kf = k.float().unsqueeze(0)
    vf = v.float().unsqueeze(0)
    hq, n, d = q.shape
    s = k.shape[1]
    mask = torch.zeros((1, 1, n, s), dtype=torch.float32)
    if causal:
        allowed = torch.arange(s)[None, :] <= (past_length + torch.arange(n))[:, None]
    else:
        allowed = torch.ones((n, s), dtype=torch.bool)
        allowed[:, past_length:] = torch.from_numpy(np.asarray(vis, dtype=bool))
    mask[0, 0].masked_fill_(~allowed, torch.finfo(torch.float32).min)
    out = torch.nn.functional.scaled_dot_product_attention(
        qf, kf, vf, attn_mask=mask, scale=scale, enable_gqa=(hq != k.shape[0]))
    return out[0].transpose(0, 1).contiguous()
