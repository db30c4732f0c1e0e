"""GPU parity of the batched walk + compaction (ddt_accept_compact_batched): every request's
accepted path, next token and compacted cache equal the single-request kernel's
(ddt_accept_compact, itself pinned to the reference's compact_tail_inplace and
follow_verified_tree golden vectors), bit-exact, with per-request budgets, prefixes and cache
capacities in one launch."""
import numpy as np
import pytest
import torch

from mdflash_b200 import kernels as K

pytestmark = pytest.mark.gpu
L, V, HEADS, D, LAYERS = 15, 1000, 2, 128, 3


def _deep_posterior(parents, ids, n, rng):
    """A posterior whose walk follows the root -> deepest-node path (then stops)."""
    depth = np.zeros(n, np.int64)
    for i in range(1, n):
        depth[i] = depth[parents[i]] + 1
    path = [int(np.argmax(depth))]
    while path[-1] != 0:
        path.append(int(parents[path[-1]]))
    path = path[::-1]
    post = rng.integers(V, 2 * V, n)  # tokens no node carries: the walk stops there
    for a, b in zip(path[:-1], path[1:]):
        post[a] = ids[b - 1]
    return post, len(path)


@pytest.mark.parametrize("seed", [0, 1])
def test_batched_walk_and_compaction_match_single(cuda_device, seed):
    dev = cuda_device
    rng = np.random.default_rng(seed)
    budgets = [1, 16, 64, 128, 256, 40, 0, 200]
    pasts = [int(x) for x in rng.integers(0, 3000, len(budgets))]
    R = len(budgets)
    logits = torch.from_numpy(rng.standard_normal((R, L, V)).astype(np.float32) * 3)
    logits[:, :, 7] += 6.0  # one likely token per depth: deep trees
    logits = logits.to(torch.bfloat16).to(dev)
    trees = K.TreeBatch.allocate(dev, budgets, L, V)
    trees.starts.copy_(torch.tensor(pasts))
    K.topk_tree_batched(logits, trees)
    torch.cuda.synchronize()
    mn = trees.max_budget + 1
    post = torch.zeros((R, mn), dtype=torch.int64)
    want_len = []
    for r in range(R):
        t = trees.tree(r)
        n = t.n_nodes
        par = t.parents[:n].cpu().numpy()
        ids = t.node_token_ids[:max(n - 1, 1)].cpu().numpy()
        p, k = _deep_posterior(par, ids, n, rng) if r % 3 else (rng.integers(0, V, n), None)
        post[r, :n] = torch.from_numpy(np.asarray(p, np.int64))
        want_len.append(k)
    post = post.to(dev)
    caches, clones = [], []
    for r in range(R):
        cap = pasts[r] + budgets[r] + 1 + int(rng.integers(0, 40)) * 8
        ts = [torch.randn((HEADS, cap, D), device=dev).to(torch.bfloat16) for _ in range(2 * LAYERS)]
        caches.append(ts)
        clones.append([x.clone() for x in ts])
    kvb = K.KvBatch([K.KvTable(ts) for ts in caches])
    acc, nacc, nxt = K.accept_compact_batched(post, trees, kvb, pasts)
    torch.cuda.synchronize()
    K.check_status(K.attention_status(dev), "ddt_accept_compact_batched")
    for r in range(R):
        t = trees.tree(r)
        a1, n1, x1 = K.accept_compact(post[r, :t.n_nodes], t, K.KvTable(clones[r]), pasts[r])
        torch.cuda.synchronize()
        k = int(n1.item())
        assert int(nacc[r].item()) == k and int(nxt[r].item()) == int(x1.item())
        assert torch.equal(acc[r, :k], a1[:k])
        if want_len[r] is not None:
            assert k == want_len[r]
        for x, y in zip(caches[r], clones[r]):
            assert torch.equal(x, y)
