"""GPU parity of the batched tree build (ddt_topk_tree_batched): every request's tree is the
reference's build_ddtree_tree (ddtree.py:84-166) for that request, bit-exact.

* Golden vectors: the reference's own trees of the tree cases, built as requests of one
  batch per (depths, vocabulary, dtype), with per-request budgets, roots and starts.
* Against the single-request kernel (ddt_topk_tree, itself pinned to the golden vectors) on
  a mix of requests with budgets from 0 to 1024, repeated launches, and a budget above the
  batch's maximum (clamped to it).
"""
from collections import defaultdict

import numpy as np
import pytest
import torch

import inputs as gin
from mdflash_b200 import kernels as K

pytestmark = pytest.mark.gpu


def _check_request(trees, r, g_ids, g_depths, g_parents, g_vis, root, start):
    cnt = int(trees.node_count[r].item())
    assert cnt == g_ids.size
    np.testing.assert_array_equal(trees.node_token_ids[r, :cnt].cpu().numpy(), g_ids)
    np.testing.assert_array_equal(trees.node_depths[r, :cnt].cpu().numpy(), g_depths)
    np.testing.assert_array_equal(trees.parents[r, :cnt + 1].cpu().numpy(), g_parents)
    n = cnt + 1
    bits = trees.anc_bits[r, :n].cpu().numpy().view(np.uint32)
    got = np.unpackbits(bits.view(np.uint8), axis=-1, bitorder="little").astype(bool)
    assert not got[:, n:].any()  # no bit past the tree, in any word of the row
    np.testing.assert_array_equal(got[:, :n], g_vis)
    ids = trees.verify_ids[r, :n].cpu().numpy()
    pos = trees.verify_pos[r, :n].cpu().numpy()
    assert ids[0] == root and pos[0] == start
    np.testing.assert_array_equal(ids[1:], g_ids)
    np.testing.assert_array_equal(pos[1:], g_depths + start)


def _groups():
    by = defaultdict(list)
    for spec in gin.TREE_CASES:
        if spec["L"] > 0:
            by[(spec["L"], spec["V"], spec["dtype"])].append(spec)
    return list(by.values())


@pytest.mark.parametrize("group", _groups(), ids=lambda g: "+".join(s["name"] for s in g))
def test_batched_tree_matches_reference(golden, cuda_device, group):
    dev = cuda_device
    logits = torch.stack([gin.tree_logits(s) for s in group]).to(dev)
    budgets = [s["budget"] for s in group]
    trees = K.TreeBatch.allocate(dev, budgets, group[0]["L"], group[0]["V"])
    roots = [1000 + 17 * r for r in range(len(group))]
    starts = [50 + 300 * r for r in range(len(group))]
    trees.root_tokens.copy_(torch.tensor(roots))
    trees.starts.copy_(torch.tensor(starts))
    K.topk_tree_batched(logits, trees)
    torch.cuda.synchronize()
    for r, spec in enumerate(group):
        name = spec["name"]
        g_par = golden[f"{name}/parents"]
        n = g_par.shape[0]
        vis = np.unpackbits(golden[f"{name}/visibility"], axis=-1, count=n).astype(bool)
        _check_request(trees, r, golden[f"{name}/node_ids"], golden[f"{name}/depths"], g_par,
                       vis, roots[r], starts[r])
        assert trees.tree(r).n_nodes == n


def _single(logits_r, budget, root, start, dev):
    t = K.topk_tree(logits_r, budget, torch.tensor([root], device=dev), start)
    n = int(t.node_count.item()) + 1
    bits = t.anc_bits[:n].cpu().numpy().view(np.uint32)
    vis = np.unpackbits(bits.view(np.uint8), axis=-1, bitorder="little", count=n).astype(bool)
    return (t.node_token_ids[:n - 1].cpu().numpy(), t.node_depths[:n - 1].cpu().numpy(),
            t.parents[:n].cpu().numpy(), vis)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_batched_tree_matches_single_requests(cuda_device, dtype):
    dev = cuda_device
    L, V = 15, gin.V_QWEN3
    budgets = [64, 0, 512, 1, 256, 1024, 128, 7, 512, 300, 64, 256]
    g = torch.Generator().manual_seed(5)
    logits = (torch.randn((len(budgets), L, V), generator=g) * 3).to(dtype)
    logits[3, :, 77] = 40.0  # a request whose drafter is sure at every depth
    logits[6] = logits[2]    # the same logits as request 2 under another budget
    logits = logits.to(dev)
    trees = K.TreeBatch.allocate(dev, budgets, L, V)
    roots = [int(x) for x in torch.randint(0, V, (len(budgets),), generator=g)]
    starts = [int(x) for x in torch.randint(0, 40000, (len(budgets),), generator=g)]
    trees.root_tokens.copy_(torch.tensor(roots))
    trees.starts.copy_(torch.tensor(starts))
    for _ in range(3):  # the workspace counters reset themselves between launches
        K.topk_tree_batched(logits, trees)
    torch.cuda.synchronize()
    for r, b in enumerate(budgets):
        ids, depths, par, vis = _single(logits[r], b, roots[r], starts[r], dev)
        _check_request(trees, r, ids, depths, par, vis, roots[r], starts[r])


def test_batched_tree_small_vocab_and_clamped_budget(cuda_device):
    """Vocabulary of 1001 fp32 logits (rows not a whole number of 16-byte vectors), budgets
    above the vocabulary, and a device budget above the batch maximum (clamped to it)."""
    dev = cuda_device
    L, V = 6, 1001
    budgets = [40, 1000, 5, 200]
    g = torch.Generator().manual_seed(9)
    logits = (torch.randn((len(budgets), L, V), generator=g) * 2).to(dev)
    trees = K.TreeBatch.allocate(dev, budgets, L, V)
    trees.budgets_dev[2] = 5000  # clamped to max_budget (1000)
    K.topk_tree_batched(logits, trees)
    torch.cuda.synchronize()
    for r, b in enumerate(budgets):
        b = 1000 if r == 2 else b
        ids, depths, par, vis = _single(logits[r], b, 0, 0, dev)
        _check_request(trees, r, ids, depths, par, vis, 0, 0)
