"""End-to-end GPU parity of the drop-in path against the reference path.

Reference path: transformers Qwen3 with attn_implementation="sdpa", a DynamicCache, and the
oracle's build_ddtree_tree / compile_ddtree_tree (the reference functions restated), exactly
as ddtree_generate calls them (ddtree.py:440-486).  Our paths: (1) the drop-in functions of
mdflash_b200.ddtree with the "ddtree_tree" attention plug-in, (2) TreeVerifier (device
resident) over transformers, (3) TreeVerifier over the fused runner.  Tree topology,
accepted paths and compaction are bit-exact; logits / KV rows are within bf16 tolerance
(max |err| / max |ref| <= 2e-2, and element-wise, relative with the row RMS as floor, within
2e-2 or within 1.25x the distance between transformers' own eager and sdpa attentions),
and the greedy posteriors agree on >= 99.9% of the rows whose reference top-1 / top-2 gap
exceeds 4 bf16 steps of the largest logit (near-ties are logged).
"""
import numpy as np
import pytest
import torch

import inputs as gin
import oracle
from mdflash_b200 import attention as A
from mdflash_b200 import ddtree as D
from mdflash_b200 import kernels as K
from mdflash_b200.cache import TreeKVCache
from mdflash_b200.verifier import TreeVerifier
from parity_util import elem_rel_err, posterior_agreement

pytestmark = pytest.mark.gpu
TOL = 2e-2
V, P, BUDGET, DEPTHS = 2048, 96, 24, 4


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)).item()


def _agreement(label, post, s):
    ref = s["ref_logits"].float()
    top2 = torch.topk(ref, 2, dim=-1).values
    tie_gap = 4 * 2.0 ** -7 * ref.abs().max().item()
    return posterior_agreement(label, post.cpu().numpy(), s["ref_post"].cpu().numpy(),
                               (top2[:, 0] - top2[:, 1]).cpu().numpy(), tie_gap)


@pytest.fixture(scope="module")
def setup(cuda_device):
    from transformers import DynamicCache, Qwen3Config, Qwen3ForCausalLM
    A.register()
    cfg = Qwen3Config(vocab_size=V, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                      rope_theta=1e6, max_position_embeddings=4096, rms_norm_eps=1e-6,
                      tie_word_embeddings=False, initializer_range=0.2,
                      attn_implementation="sdpa")
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg).to(cuda_device, torch.bfloat16).eval()
    rng = np.random.default_rng(7)
    ids = torch.from_numpy(rng.integers(0, V, (1, P))).to(cuda_device)
    logits = torch.from_numpy(rng.standard_normal((DEPTHS, V)).astype(np.float32) * 3).to(
        torch.bfloat16)
    # ---- reference path ----
    model.config._attn_implementation = "sdpa"
    ref_cache = DynamicCache()
    with torch.inference_mode():
        out = model(ids, position_ids=torch.arange(P, device=cuda_device)[None],
                    past_key_values=ref_cache, use_cache=True)
        root = out.logits[0, -1].argmax()
        tree = oracle.build_ddtree_tree(logits, BUDGET)
        node_ids, depths, parents, child_maps, vis, _ = tree
        n = 1 + node_ids.numel()
        vib = torch.empty((1, n), dtype=torch.long, device=cuda_device)
        vpb = torch.empty((1, n), dtype=torch.long, device=cuda_device)
        amb = torch.zeros((1, 1, n, P + n), dtype=torch.bfloat16, device=cuda_device)
        tvb = torch.empty((n, n), dtype=torch.bool, device=cuda_device)
        vi, vp, am, _, _ = oracle.compile_ddtree_tree(root, P, node_ids, depths, vis, P,
                                                      torch.bfloat16, cuda_device, vib, vpb, amb,
                                                      tvb, 0, 0)
        prefix = [(l.keys.clone(), l.values.clone()) for l in ref_cache.layers]
        ref_logits = model(vi, position_ids=vp, attention_mask=am, past_key_values=ref_cache,
                           use_cache=True).logits[0]
        # transformers' eager attention on the same prefix: the spread of the reference's own
        # bf16 implementations, the yardstick of the element-wise check
        eager_cache = DynamicCache()
        for li, (k, v) in enumerate(prefix):
            eager_cache.update(k, v, li)
        model.config._attn_implementation = "eager"
        eager_logits = model(vi, position_ids=vp, attention_mask=am, past_key_values=eager_cache,
                             use_cache=True).logits[0]
        model.config._attn_implementation = "sdpa"
    ref_post = ref_logits.argmax(-1)
    ref_acc, ref_next = oracle.follow_verified_tree(child_maps, ref_post.cpu())
    return dict(model=model, ids=ids, logits=logits, root=root, tree=tree, n=n,
                ref_logits=ref_logits, elem_bound=max(TOL, 1.25 * elem_rel_err(eager_logits,
                                                                               ref_logits)), ref_post=ref_post, ref_cache=ref_cache, ref_acc=ref_acc,
                ref_next=ref_next, vi=vi, vp=vp)


def test_dropin_functions_and_plugin(setup, cuda_device):
    from transformers import DynamicCache
    s = setup
    model = s["model"]
    model.config._attn_implementation = A.ATTN_IMPLEMENTATION
    cache = DynamicCache()
    with torch.inference_mode():
        out = model(s["ids"], position_ids=torch.arange(P, device=cuda_device)[None],
                    past_key_values=cache, use_cache=True)  # causal prefill on our kernel
        for lo, lr in zip(cache.layers, s["ref_cache"].layers):
            assert _rel(lo.keys, lr.keys[..., :P, :]) <= TOL
            assert _rel(lo.values, lr.values[..., :P, :]) <= TOL
        root = out.logits[0, -1].argmax()
        node_ids, depths, parents, child_maps, vis, sub = D.build_ddtree_tree(
            s["logits"].to(cuda_device), BUDGET)
        o_ids, o_depths, o_par, o_cm, o_vis, _ = s["tree"]
        assert torch.equal(node_ids, o_ids) and torch.equal(depths, o_depths)
        assert parents == o_par and child_maps == o_cm and torch.equal(vis, o_vis)
        assert set(sub) == set(D.DDTREE_TREE_BUILD_STAGE_ORDER)
        n = s["n"]
        vib = torch.empty((1, n), dtype=torch.long, device=cuda_device)
        vpb = torch.empty((1, n), dtype=torch.long, device=cuda_device)
        amb = torch.zeros((1, 1, n, P + n), dtype=torch.bfloat16, device=cuda_device)
        tvb = torch.empty((n, n), dtype=torch.bool, device=cuda_device)
        vi, vp, am, pl, cl = D.compile_ddtree_tree(root, P, node_ids, depths, vis, P,
                                                   torch.bfloat16, cuda_device, vib, vpb, amb, tvb,
                                                   0, 0)
        assert torch.equal(vi, s["vi"]) and torch.equal(vp, s["vp"]) and (pl, cl) == (P, n)
        logits = model(vi, position_ids=vp, attention_mask=am, past_key_values=cache,
                       use_cache=True).logits[0]
        assert _rel(logits, s["ref_logits"]) <= TOL
        assert elem_rel_err(logits, s["ref_logits"]) <= s["elem_bound"]
        post = logits.argmax(-1)
        assert _agreement("e2e drop-in", post, s) >= 0.999
        acc, nxt = D.follow_verified_tree(child_maps, post[None])
        acc_host, nxt_host = oracle.follow_verified_tree(child_maps, post.cpu())
        assert (acc, nxt) == (acc_host, nxt_host)
        # forced deep path: compaction through the drop-in on both caches, bit-exact
        forced = gin.follow_posterior(dict(kind="path", target=-1, seed=3, V=V),
                                      node_ids.numpy(), np.asarray(parents, np.int32))
        f_acc, f_next = D.follow_verified_tree(child_maps, torch.from_numpy(forced).to(cuda_device)[None])
        assert (f_acc, f_next) == oracle.follow_verified_tree(child_maps, forced)
        before = [(l.keys.float().cpu().numpy().copy(), l.values.float().cpu().numpy().copy())
                  for l in cache.layers]
        D.compact_dynamic_cache(cache, P, f_acc)
        for layer, (kb, vb) in zip(cache.layers, before):
            assert layer.keys.shape[-2] == P + len(f_acc)
            np.testing.assert_array_equal(layer.keys.float().cpu().numpy(),
                                          oracle.compact_rows(kb, P, f_acc))
            np.testing.assert_array_equal(layer.values.float().cpu().numpy(),
                                          oracle.compact_rows(vb, P, f_acc))
    A.clear_tree_context()


def test_compact_tail_inplace_mirrors_reference_checks(cuda_device):
    mod = D.load_cpp_compact_module()
    t = torch.randn((1, 2, 12, 128), device=cuda_device).to(torch.bfloat16)
    before = t.float().cpu().numpy().copy()
    keep = torch.tensor([0, 2, 5], device=cuda_device)
    mod.compact_tail_inplace(t, 4, keep)
    np.testing.assert_array_equal(t.float().cpu().numpy()[..., :7, :],
                                  oracle.compact_rows(before, 4, [0, 2, 5]))
    with pytest.raises(RuntimeError, match="keep_count exceeds"):
        mod.compact_tail_inplace(t, 10, torch.tensor([0, 1, 2], device=cuda_device))
    with pytest.raises(RuntimeError, match="dtype torch.long"):
        mod.compact_tail_inplace(t, 4, keep.to(torch.int32))


@pytest.mark.parametrize("fused", [False, True])
def test_tree_verifier_matches_reference(setup, cuda_device, fused):
    s = setup
    model = s["model"]
    model.config._attn_implementation = A.ATTN_IMPLEMENTATION
    cache = TreeKVCache(2, P + BUDGET + 8).allocate(2, 128, torch.bfloat16, cuda_device)
    verifier = TreeVerifier(model, cache, BUDGET, DEPTHS, V, cuda_device, keep_logits=True,
                            fused=fused)
    with torch.inference_mode():
        if fused:
            pos = torch.arange(P, device=cuda_device)
            verifier.runner.forward(s["ids"][0], pos, cache, 0, None, causal=True)
        else:
            model(s["ids"], position_ids=torch.arange(P, device=cuda_device)[None],
                  past_key_values=cache, use_cache=True)
        for lo, lr in zip(cache.layers, s["ref_cache"].layers):
            assert _rel(lo.keys, lr.keys[..., :P, :]) <= TOL
        res = verifier.step(s["logits"].to(cuda_device), s["root"].view(1), P)
        torch.cuda.synchronize()
    o_ids, o_depths, o_par, _, _, _ = s["tree"]
    n = s["n"]
    assert res.n_nodes == n
    assert verifier.tree.parents[:n].tolist() == o_par
    assert torch.equal(verifier.tree.node_token_ids[:n - 1].cpu(), o_ids)
    assert _rel(res.logits, s["ref_logits"]) <= TOL
    assert elem_rel_err(res.logits, s["ref_logits"]) <= s["elem_bound"]
    assert _agreement("e2e verifier fused" if fused else "e2e verifier", res.posterior, s) >= 0.999
    k = int(res.n_accepted.item())
    acc = res.accepted[:k].tolist()
    o_acc, o_next = oracle.follow_verified_tree((np.asarray(o_par, np.int32), o_ids.numpy()),
                                                res.posterior.cpu())
    assert acc == o_acc and int(res.next_token.item()) == o_next
    if torch.equal(res.posterior, s["ref_post"]):
        assert acc == s["ref_acc"]
    verifier.commit(P, k)
    assert cache.get_seq_length() == P + k


def test_tree_verifier_fused_lm_head(setup, cuda_device):
    """The fused runner with the fused lm_head -> argmax kernel (no logits): same tree, the
    posterior within the reference's near-ties, and the walk of that posterior."""
    s = setup
    model = s["model"]
    cache = TreeKVCache(2, P + BUDGET + 8).allocate(2, 128, torch.bfloat16, cuda_device)
    verifier = TreeVerifier(model, cache, BUDGET, DEPTHS, V, cuda_device, fused=True,
                            fused_head=True)
    with torch.inference_mode():
        verifier.runner.forward(s["ids"][0], torch.arange(P, device=cuda_device), cache, 0, None,
                                causal=True)
        res = verifier.step(s["logits"].to(cuda_device), s["root"].view(1), P)
        torch.cuda.synchronize()
    o_ids, o_depths, o_par, _, _, _ = s["tree"]
    assert res.n_nodes == s["n"] and res.logits is None
    verifier.check()
    assert _agreement("e2e verifier fused lm_head", res.posterior, s) >= 0.999
    k = int(res.n_accepted.item())
    o_acc, o_next = oracle.follow_verified_tree((np.asarray(o_par, np.int32), o_ids.numpy()),
                                                res.posterior.cpu())
    assert res.accepted[:k].tolist() == o_acc and int(res.next_token.item()) == o_next


def test_follow_verified_tree_on_a_foreign_tree(setup, cuda_device):
    """child_maps that are not the tree build_ddtree_tree just built (here: the oracle's tree
    of other logits) are walked on the device too, with the reference's result."""
    s = setup
    D.build_ddtree_tree(s["logits"].to(cuda_device), BUDGET)  # registers a different tree
    other = gin.tree_logits(gin.TREE_CASES[7])  # ties_v50_b10: V = 50, 4 depths
    node_ids, depths, parents, child_maps, vis, _ = oracle.build_ddtree_tree(other, 10)
    par = np.asarray(parents, np.int32)
    for kind, seed in (("path", 1), ("random", 2), ("none", 3)):
        spec = dict(kind=kind, target=-1, seed=seed, V=50)
        post = gin.follow_posterior(spec, node_ids.numpy(), par)
        got = D.follow_verified_tree(child_maps, torch.from_numpy(post).to(cuda_device)[None])
        assert got == oracle.follow_verified_tree(child_maps, post), kind


def test_tree_verifier_context_features(setup, cuda_device):
    """feature_layers: the step returns the drafter's context features of the accepted rows,
    extract_context_feature(output.hidden_states, layer_ids).index_select(1, accepted)
    (model/utils.py:17-26, ddtree.py:487), here with layer ids -1 (the embeddings), 0 (the
    residual stream after layer 0) and 1 (the last layer: the final normed state).  Against
    transformers' own hidden_states of the same tree on the same prefix (through the plug-in),
    within the bf16 tolerance; the gathered rows are exactly the accepted rows."""
    from mdflash_b200.runner import Qwen3VerifyRunner
    s = setup
    dev = cuda_device
    model = s["model"]
    model.config._attn_implementation = A.ATTN_IMPLEMENTATION
    layers = [-1, 0, 1]
    runner = Qwen3VerifyRunner(model)
    caches = [TreeKVCache(2, P + BUDGET + 8).allocate(2, 128, torch.bfloat16, dev)
              for _ in range(2)]
    with torch.inference_mode():
        for c in caches:
            runner.forward(s["ids"][0], torch.arange(P, device=dev), c, 0, None, causal=True)
        ver = TreeVerifier(model, caches[0], BUDGET, DEPTHS, V, dev, fused=True, runner=runner,
                           feature_layers=layers)
        res = ver.step(s["logits"].to(dev), s["root"].view(1), P)
        tree, n = ver.tree, res.n_nodes
        with A.tree_verify(tree, P, n, status=ver.status):
            out = model(tree.verify_ids[:n].view(1, n),
                        position_ids=tree.verify_pos[:n].view(1, n),
                        past_key_values=caches[1], use_cache=True, output_hidden_states=True)
    torch.cuda.synchronize()
    ver.check()
    H = model.config.hidden_size
    ref = torch.cat([out.hidden_states[lid + 1][0] for lid in layers], dim=-1)
    for j, lid in enumerate(layers):
        a, b = ver.features[:n, j * H:(j + 1) * H], ref[:, j * H:(j + 1) * H]
        print(f"[features] layer {lid}: rel {_rel(a, b):.2e}, elem {elem_rel_err(a, b):.2e}")
        assert _rel(a, b) <= TOL and elem_rel_err(a, b) <= TOL
    k = int(res.n_accepted.item())
    acc = res.accepted[:k]
    assert torch.equal(res.target_hidden[:k], ver.features[:n].index_select(0, acc))
