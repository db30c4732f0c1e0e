"""Pin the CPU oracle against the golden vectors produced by the reference's own code.

These run without a GPU.  The oracle is then trusted as the checker of the CUDA path.
"""
import numpy as np
import pytest
import torch

import inputs as gin
import oracle


def _tree(golden, name):
    return (golden[f"{name}/node_ids"], golden[f"{name}/depths"], golden[f"{name}/parents"])


@pytest.mark.parametrize("spec", gin.TREE_CASES, ids=[c["name"] for c in gin.TREE_CASES])
def test_heap_matches_reference_given_reference_logprobs(golden, spec):
    """Best-first heap (ddtree.py:116-147) fed with the reference's own top log-probs
    reproduces the reference topology bit for bit."""
    name = spec["name"]
    ids, depths, parents = _tree(golden, name)
    if spec["budget"] <= 0 or spec["L"] == 0:
        assert ids.size == 0 and parents.tolist() == [-1]
        return
    o_ids, o_depths, o_parents = oracle.build_tree(golden[f"{name}/top_lp"],
                                                   golden[f"{name}/top_ids"], spec["budget"])
    np.testing.assert_array_equal(o_ids, ids)
    np.testing.assert_array_equal(o_depths, depths)
    np.testing.assert_array_equal(o_parents, parents)


@pytest.mark.parametrize("spec", gin.TREE_CASES, ids=[c["name"] for c in gin.TREE_CASES])
def test_logz_topk_matches_reference(golden, spec):
    """Top-k ids equal the reference's (canonical tie order); log Z (double accumulate,
    one rounding) is within 2 float ulps of torch.logsumexp; log-probs likewise."""
    name = spec["name"]
    if spec["budget"] <= 0 or spec["L"] == 0:
        return
    k = min(spec["budget"], spec["V"])
    top_lp, top_ids, logz = oracle.logz_topk(gin.tree_logits(spec), k)
    np.testing.assert_array_equal(top_ids, golden[f"{name}/top_ids"])
    ref_lz = golden[f"{name}/logz"]
    ulps = np.abs(logz.view(np.int32).astype(np.int64) - ref_lz.view(np.int32).astype(np.int64))
    assert ulps.max() <= 2, ulps
    np.testing.assert_allclose(top_lp, golden[f"{name}/top_lp"], rtol=0, atol=4e-6)


@pytest.mark.parametrize("spec", gin.TREE_CASES, ids=[c["name"] for c in gin.TREE_CASES])
def test_build_ddtree_tree_end_to_end(golden, spec):
    """Whole build_ddtree_tree (ddtree.py:84-166): same return types and, on every seeded
    case here, the same topology and visibility as the reference."""
    name = spec["name"]
    node_ids, depths, parents, child_maps, vis, sub = oracle.build_ddtree_tree(
        gin.tree_logits(spec), spec["budget"])
    g_ids, g_depths, g_parents = _tree(golden, name)
    assert node_ids.dtype == torch.long and depths.dtype == torch.long
    assert isinstance(parents, list) and isinstance(child_maps, list)
    np.testing.assert_array_equal(node_ids.numpy(), g_ids)
    np.testing.assert_array_equal(depths.numpy(), g_depths)
    assert parents == g_parents.tolist()
    n = len(parents)
    g_vis = np.unpackbits(golden[f"{name}/visibility"], axis=-1, count=n).astype(bool)
    np.testing.assert_array_equal(vis.numpy(), g_vis)
    assert set(sub) == {"tree_build_copy", "tree_build_heap", "tree_build_visibility"}


@pytest.mark.parametrize("spec", gin.TREE_CASES, ids=[c["name"] for c in gin.TREE_CASES])
def test_ancestor_bits_equal_visibility(golden, spec):
    name = spec["name"]
    parents = golden[f"{name}/parents"]
    n = parents.shape[0]
    bits = oracle.ancestor_bits(parents)
    g_vis = np.unpackbits(golden[f"{name}/visibility"], axis=-1, count=n).astype(bool)
    unpacked = np.unpackbits(bits.view(np.uint8), axis=-1, bitorder="little", count=n).astype(bool)
    np.testing.assert_array_equal(unpacked, g_vis)


@pytest.mark.parametrize("spec", gin.COMPILE_CASES, ids=[c["name"] for c in gin.COMPILE_CASES])
def test_compile_matches_reference(golden, spec):
    tree = spec["tree"]
    node_ids = torch.from_numpy(golden[f"{tree}/node_ids"])
    depths = torch.from_numpy(golden[f"{tree}/depths"])
    parents = golden[f"{tree}/parents"]
    n = parents.shape[0]
    vis = torch.from_numpy(np.unpackbits(golden[f"{tree}/visibility"], axis=-1, count=n)
                           .astype(bool))
    dtype = getattr(torch, spec["dtype"])
    cap, past = spec["cap"], spec["past"]
    ids_buf = torch.full((1, cap), -7, dtype=torch.long)
    pos_buf = torch.full((1, cap), -7, dtype=torch.long)
    mask_buf = torch.zeros((1, 1, cap, past + cap + 8), dtype=dtype)
    if spec["prev_len"] > 0:
        mask_buf[0, 0, :spec["prev_len"],
                 spec["prev_start"]:spec["prev_start"] + spec["prev_len"]] = torch.finfo(dtype).min
    vis_buf = torch.zeros((cap, cap), dtype=torch.bool)
    ids, pos, mask, pl, cl = oracle.compile_ddtree_tree(
        torch.tensor(spec["root"]), spec["start"], node_ids, depths, vis, past, dtype, None,
        ids_buf, pos_buf, mask_buf, vis_buf, spec["prev_start"], spec["prev_len"])
    name = spec["name"]
    np.testing.assert_array_equal(ids.numpy(), golden[f"{name}/ids"])
    np.testing.assert_array_equal(pos.numpy(), golden[f"{name}/pos"])
    np.testing.assert_array_equal(mask.float().numpy(), golden[f"{name}/mask"])
    np.testing.assert_array_equal(mask_buf.float().numpy(), golden[f"{name}/mask_buffer"])
    assert [pl, cl] == golden[f"{name}/lengths"].tolist()


@pytest.mark.parametrize("spec", gin.FOLLOW_CASES, ids=[c["name"] for c in gin.FOLLOW_CASES])
def test_follow_matches_reference(golden, spec):
    tree = spec["tree"]
    node_ids = golden[f"{tree}/node_ids"]
    parents = golden[f"{tree}/parents"]
    post = gin.follow_posterior(spec, node_ids, parents)
    np.testing.assert_array_equal(post, golden[f"{spec['name']}/posterior"])
    acc, nxt = oracle.follow_verified_tree((parents, node_ids), post)
    assert acc == golden[f"{spec['name']}/accepted"].tolist()
    assert nxt == int(golden[f"{spec['name']}/next_token"][0])


def test_follow_forced_paths_accept_beyond_root(golden):
    deep = golden["follow_deepest/accepted"]
    assert deep.size >= 3 and np.all(np.diff(deep) > 0)
    assert golden["follow_deepest_b1024/accepted"].size >= 4


@pytest.mark.parametrize("spec", gin.COMPACT_CASES, ids=[c["name"] for c in gin.COMPACT_CASES])
def test_compaction_matches_reference(golden, spec):
    layers = gin.compact_cache(spec)
    out = oracle.compact_dynamic_cache(layers, spec["past"], list(spec["keep"]))
    name = spec["name"]
    for li, (k, v) in enumerate(out):
        np.testing.assert_array_equal(k, golden[f"{name}/k{li}"])
        np.testing.assert_array_equal(v, golden[f"{name}/v{li}"])
        assert k.shape[-2] == int(golden[f"{name}/seq_len"][0])


def test_argmax_tie_rule():
    x = np.array([[1.0, 3.0, 3.0, 2.0], [np.nan, 5.0, np.nan, 1.0], [-1, -1, -1, -1]], np.float32)
    assert oracle.argmax(x).tolist() == [1, 0, 0]
    assert oracle.argmax(x).tolist() == torch.argmax(torch.from_numpy(x), -1).tolist()


@pytest.mark.parametrize("spec", gin.ATTN_CASES, ids=[c["name"] for c in gin.ATTN_CASES])
def test_tree_attention_oracle_matches_reference(golden, spec):
    q, k, v, parents = gin.attn_inputs(spec)
    np.testing.assert_array_equal(parents, golden[f"{spec['name']}/parents"])
    vis = oracle.visibility(parents)
    out = oracle.tree_attention(q, k, v, vis, spec["past"])
    np.testing.assert_allclose(out.numpy(), golden[f"{spec['name']}/out"], rtol=1e-5, atol=1e-6)


def test_random_tree_shape():
    p = gin.random_tree(513, 7)
    assert p[0] == -1 and np.all(p[1:] < np.arange(1, 513))
    depth = np.zeros(513, np.int64)
    for i in range(1, 513):
        depth[i] = depth[p[i]] + 1
    assert depth.max() <= 16


@pytest.mark.parametrize("spec", gin.SAMPLED_CASES, ids=[c["name"] for c in gin.SAMPLED_CASES])
def test_sampled_candidate_tree_matches_reference(golden, spec):
    """build_sampled_candidate_tree (ddtree.py:169-224) restated: topology, tokens, depths and
    visibility equal the reference's on chains with shared prefixes, budget cuts in the middle
    of a chain, identical chains and the empty cases."""
    name = spec["name"]
    node_ids, depths, parents, child_maps, vis = oracle.build_sampled_candidate_tree(
        gin.sampled_chains(spec), spec["budget"])
    np.testing.assert_array_equal(node_ids.numpy(), golden[f"{name}/node_ids"])
    np.testing.assert_array_equal(depths.numpy(), golden[f"{name}/depths"])
    assert parents == golden[f"{name}/parents"].tolist()
    n = len(parents)
    g_vis = np.unpackbits(golden[f"{name}/visibility"], axis=-1, count=n).astype(bool)
    np.testing.assert_array_equal(vis.numpy(), g_vis)
    for i in range(1, n):
        assert child_maps[parents[i]][int(node_ids[i - 1])] == i


def test_greedy_chains_are_the_argmax_chain(golden):
    spec = gin.GREEDY_CHAIN_CASE
    logits = gin._logits(spec["seed"], spec["L"], spec["V"], "normal3")
    chains = golden["greedy_chains/chains"]
    assert chains.shape == (spec["S"], spec["L"])
    np.testing.assert_array_equal(chains, np.tile(oracle.argmax(logits), (spec["S"], 1)))
