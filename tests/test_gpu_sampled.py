"""GPU parity of the sampled-tree path of the MDFlash / P-Express variants:
ddt_chain_tree against build_sampled_candidate_tree (ddtree.py:169-224, golden vectors
from the reference and the oracle restatement; bit-exact), and ddt_sample_chains against
sample_candidate_chains (mdflash.py:19-40: exact at temperature 0, and the sampling
distribution of softmax(logits / T) by a chi-square test otherwise)."""
import numpy as np
import pytest
import torch

import inputs as gin
import oracle
from mdflash_b200 import ddtree as D
from mdflash_b200 import kernels as K
from mdflash_b200 import mdflash as M

pytestmark = pytest.mark.gpu


def _check_tree(tree, o_ids, o_depths, o_par, o_vis, root=None, start=0):
    n = len(o_par)
    assert int(tree.node_count.item()) == n - 1
    np.testing.assert_array_equal(tree.parents[:n].cpu().numpy(), np.asarray(o_par, np.int32))
    np.testing.assert_array_equal(tree.node_token_ids[:n - 1].cpu().numpy(), o_ids)
    np.testing.assert_array_equal(tree.node_depths[:n - 1].cpu().numpy(), o_depths)
    bits = tree.anc_bits[:n].cpu().numpy().view(np.uint32)
    vis = np.unpackbits(bits.view(np.uint8), axis=-1, bitorder="little", count=n).astype(bool)
    np.testing.assert_array_equal(vis, o_vis)
    ids = tree.verify_ids[:n].cpu().numpy()
    pos = tree.verify_pos[:n].cpu().numpy()
    assert pos[0] == start and (root is None or ids[0] == root)
    np.testing.assert_array_equal(ids[1:], o_ids)
    np.testing.assert_array_equal(pos[1:], np.asarray(o_depths) + start)


@pytest.mark.parametrize("spec", gin.SAMPLED_CASES, ids=[c["name"] for c in gin.SAMPLED_CASES])
def test_chain_tree_matches_reference(golden, cuda_device, spec):
    name = spec["name"]
    chains = gin.sampled_chains(spec)
    root = torch.tensor([77], dtype=torch.int64, device=cuda_device)
    tree = K.chain_tree(chains.to(cuda_device), spec["budget"], root_token=root, start=50)
    torch.cuda.synchronize()
    par = golden[f"{name}/parents"]
    n = par.shape[0]
    g_vis = np.unpackbits(golden[f"{name}/visibility"], axis=-1, count=n).astype(bool)
    _check_tree(tree, golden[f"{name}/node_ids"], golden[f"{name}/depths"], par, g_vis, 77, 50)


@pytest.mark.parametrize("S,L,V,budget,seed", [
    (1024, 20, 2, 1024, 1), (1024, 15, 3, 700, 2), (300, 12, 5, 1024, 3), (700, 20, 4, 513, 4),
    (1, 20, 9, 20, 5), (1024, 1, 1000, 1024, 6)])
def test_chain_tree_matches_oracle(cuda_device, S, L, V, budget, seed):
    rng = np.random.default_rng(seed)
    chains = torch.from_numpy(rng.integers(0, V, (S, L)).astype(np.int64))
    tree = K.chain_tree(chains.to(cuda_device), budget)
    torch.cuda.synchronize()
    o_ids, o_depths, o_par, _, o_vis = oracle.build_sampled_candidate_tree(chains, budget)
    _check_tree(tree, o_ids.numpy(), o_depths.numpy(), o_par, o_vis.numpy())


def test_dropin_sampled_tree_compile_and_walk(cuda_device):
    """The drop-in returns the reference's types and values; compile_ddtree_tree and
    follow_verified_tree then use the registered device tree."""
    rng = np.random.default_rng(9)
    chains = torch.from_numpy(rng.integers(0, 4, (128, 15)).astype(np.int64))
    got = D.build_sampled_candidate_tree(chains.to(cuda_device), 96)
    ref = oracle.build_sampled_candidate_tree(chains, 96)
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
    assert got[2] == ref[2] and got[3] == ref[3] and torch.equal(got[4], ref[4])
    node_ids, depths, parents, child_maps, vis = got
    n = len(parents)
    P = 40
    vib = torch.empty((1, n), dtype=torch.long, device=cuda_device)
    vpb = torch.empty((1, n), dtype=torch.long, device=cuda_device)
    amb = torch.zeros((1, 1, n, P + n), dtype=torch.bfloat16, device=cuda_device)
    tvb = torch.empty((n, n), dtype=torch.bool, device=cuda_device)
    vi, vp, am, pl, cl = D.compile_ddtree_tree(torch.tensor(5), P, node_ids, depths, vis, P,
                                               torch.bfloat16, cuda_device, vib, vpb, amb, tvb,
                                               0, 0)
    o_vi, o_vp, o_am, _, _ = oracle.compile_ddtree_tree(
        torch.tensor(5), P, node_ids, depths, vis, P, torch.bfloat16, None,
        torch.empty((1, n), dtype=torch.long), torch.empty((1, n), dtype=torch.long),
        torch.zeros((1, 1, n, P + n), dtype=torch.bfloat16), torch.empty((n, n), dtype=torch.bool),
        0, 0)
    assert torch.equal(vi.cpu(), o_vi) and torch.equal(vp.cpu(), o_vp)
    assert torch.equal(am.cpu().float(), o_am.float()) and cl == n
    post = gin.follow_posterior(dict(kind="path", target=-1, seed=3, V=4), node_ids.numpy(),
                                np.asarray(parents, np.int32))
    acc = D.follow_verified_tree(child_maps, torch.from_numpy(post).to(cuda_device)[None])
    assert acc == oracle.follow_verified_tree(child_maps, post)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sample_chains_greedy_matches_reference(golden, cuda_device, dtype):
    spec = gin.GREEDY_CHAIN_CASE
    logits = torch.from_numpy(gin._logits(spec["seed"], spec["L"], spec["V"], "normal3"))
    chains = M.sample_candidate_chains(logits.to(dtype).to(cuda_device), spec["S"], 0.0)
    torch.cuda.synchronize()
    if dtype == torch.float32:
        np.testing.assert_array_equal(chains.cpu().numpy(), golden["greedy_chains/chains"])
    else:  # the argmax of the bf16 logits, ties to the lowest index
        ref = oracle.argmax(logits.to(dtype).float().numpy())
        np.testing.assert_array_equal(chains.cpu().numpy(), np.tile(ref, (spec["S"], 1)))


@pytest.mark.parametrize("temp", [1.0, 0.5, 2.5])
def test_sample_chains_distribution(cuda_device, temp):
    """200k draws per depth from 16 tokens: every depth's counts pass a chi-square test
    against softmax(logits / T) (15 degrees of freedom, threshold at p ~ 1e-6), and the
    chains are the per-depth draws stacked."""
    g = torch.Generator().manual_seed(11)
    L, V, S = 4, 16, 200_000
    logits = torch.randn((L, V), generator=g) * 2
    chains = K.sample_chains(logits.to(cuda_device), S, temp, seed=1234, offset=7)
    torch.cuda.synchronize()
    c = chains.cpu().numpy()
    assert c.shape == (S, L) and c.min() >= 0 and c.max() < V
    probs = torch.softmax(logits.double() / temp, -1).numpy()
    for d in range(L):
        counts = np.bincount(c[:, d], minlength=V)
        expect = probs[d] * S
        chi2 = float(((counts - expect) ** 2 / expect).sum())
        assert chi2 < 55.0, (d, chi2)
    # the same (seed, offset) gives the same chains; another offset other chains
    again = K.sample_chains(logits.to(cuda_device), S, temp, seed=1234, offset=7)
    other = K.sample_chains(logits.to(cuda_device), S, temp, seed=1234, offset=8)
    assert torch.equal(again, chains) and not torch.equal(other, chains)


def test_sample_chains_full_vocabulary(cuda_device):
    """Qwen3 vocabulary, bf16 drafter logits: draws stay in range, a dominant token is drawn
    at its probability, and torch.manual_seed makes the drop-in reproducible."""
    g = torch.Generator().manual_seed(3)
    L, V, S = 15, gin.V_QWEN3, 1024
    logits = (torch.randn((L, V), generator=g) * 3)
    logits[:, 123] = 16.4  # about half of the probability mass at T = 1
    x = logits.to(torch.bfloat16).to(cuda_device)
    torch.manual_seed(5)
    a = M.sample_candidate_chains(x, S, 1.0)
    torch.manual_seed(5)
    b = M.sample_candidate_chains(x, S, 1.0)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    c = a.cpu().numpy()
    assert c.min() >= 0 and c.max() < V
    p = torch.softmax(x.float().cpu().double(), -1)[:, 123].numpy()
    frac = (c == 123).mean(0)
    assert np.all(np.abs(frac - p) < 5 * np.sqrt(p * (1 - p) / S) + 1e-3), (frac, p)
