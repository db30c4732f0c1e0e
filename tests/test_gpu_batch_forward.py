"""The verify forward of several requests at once (Qwen3VerifyRunner.forward_batch) against
each request's own forward (Qwen3VerifyRunner.forward, the path TreeVerifier runs).

* logits within the bf16 tolerance, element-wise, and the greedy posteriors equal on every
  decided row (near-ties logged); the tree rows' K/V written into each request's cache
  within the same tolerance;
* batch invariance: a request's logits are bit-identical whichever other requests share the
  batch and in whichever order, because the projections run in GEMMs of a fixed row count.
  That keeps a request's results the same at every GPU count of the request mix.
"""
import numpy as np
import pytest
import torch

from mdflash_b200 import kernels as K
from mdflash_b200.cache import TreeKVCache
from parity_util import elem_rel_err, posterior_agreement

pytestmark = pytest.mark.gpu
TOL = 2e-2
V, DEPTHS, CHUNK = 2048, 4, 128
# (prefix, budget) per request: tree rows 1 + budget (capped by the depths' top-k)
REQUESTS = [(300, 24), (40, 60), (1000, 7), (129, 33)]


@pytest.fixture(scope="module")
def model(cuda_device):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=V, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                      rope_theta=1e6, max_position_embeddings=4096, rms_norm_eps=1e-6,
                      tie_word_embeddings=False, initializer_range=0.2)
    torch.manual_seed(1)
    return Qwen3ForCausalLM(cfg).to(cuda_device, torch.bfloat16).eval()


def _request(runner, dev, prefix, budget, seed):
    """A prefilled cache and the request's device tree."""
    rng = np.random.default_rng(seed)
    cache = TreeKVCache(2, prefix + budget + 8).allocate(2, 128, torch.bfloat16, dev)
    ids = torch.from_numpy(rng.integers(0, V, prefix)).to(dev)
    with torch.inference_mode():
        runner.forward(ids, torch.arange(prefix, device=dev), cache, 0, None, causal=True)
    logits = torch.from_numpy(rng.standard_normal((DEPTHS, V)).astype(np.float32) * 3).to(
        torch.bfloat16).to(dev)
    root = torch.tensor([int(rng.integers(0, V))], device=dev)
    tree = K.topk_tree(logits, budget, root, prefix)
    return cache, tree


def _batch(runner, dev, reqs, trees, caches):
    """forward_batch over `reqs` (indices), their rows request after request, padded."""
    segs, pasts, ancs, ids, pos = [], [], [], [], []
    off = 0
    for r in reqs:
        t = trees[r]
        n = t.n_nodes
        segs.append((off, n))
        pasts.append(REQUESTS[r][0])
        ancs.append(t.anc_bits[:n])
        ids.append(t.verify_ids[:n])
        pos.append(t.verify_pos[:n])
        off += n
    t_pad = -(-off // CHUNK) * CHUNK
    ids_b = torch.zeros(t_pad, dtype=torch.int64, device=dev)
    pos_b = torch.zeros(t_pad, dtype=torch.int64, device=dev)
    ids_b[:off] = torch.cat(ids)
    pos_b[:off] = torch.cat(pos)
    with torch.inference_mode():
        logits = runner.forward_batch(ids_b, pos_b, segs, [caches[r] for r in reqs], pasts, ancs,
                                      chunk=CHUNK, lanes=2)
    return {r: logits[o:o + n].clone() for r, (o, n) in zip(reqs, segs)}


def test_forward_batch_matches_per_request_forward(cuda_device, model):
    from mdflash_b200.runner import Qwen3VerifyRunner
    dev = cuda_device
    runner = Qwen3VerifyRunner(model)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    own, trees, batch_caches = {}, [], []
    for r, (prefix, budget) in enumerate(REQUESTS):
        cache, tree = _request(runner, dev, prefix, budget, 40 + r)
        trees.append(tree)
        # the same prefilled prefix for the batched run
        twin = TreeKVCache(2, cache.capacity).allocate(2, 128, torch.bfloat16, dev)
        for la, lb in zip(cache.layers, twin.layers):
            lb.k_buf.copy_(la.k_buf)
            lb.v_buf.copy_(la.v_buf)
        twin.set_seq_length(prefix)
        batch_caches.append(twin)
        n = tree.n_nodes
        with torch.inference_mode():
            own[r] = (runner.forward(tree.verify_ids[:n], tree.verify_pos[:n], cache, prefix,
                                     tree.anc_bits[:n], status=status).clone(), cache)
    got = _batch(runner, dev, list(range(len(REQUESTS))), trees, batch_caches)
    torch.cuda.synchronize()
    K.check_status(status)
    K.check_status(K.attention_status(dev))
    for r, (prefix, budget) in enumerate(REQUESTS):
        ref, cache = own[r]
        ours = got[r]
        n = ref.shape[0]
        rel = ((ours.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
        eerr = elem_rel_err(ours, ref)
        print(f"[batch] request {r} (prefix {prefix}, {n} rows): rel {rel:.2e}, elem {eerr:.2e}")
        assert rel <= TOL and eerr <= TOL
        top2 = torch.topk(ref.float(), 2, dim=-1).values
        agree = posterior_agreement(f"batch request {r}", ours.argmax(-1).cpu().numpy(),
                                    ref.argmax(-1).cpu().numpy(),
                                    (top2[:, 0] - top2[:, 1]).cpu().numpy(),
                                    4 * 2.0 ** -7 * ref.float().abs().max().item())
        assert agree == 1.0
        for la, lb in zip(cache.layers, batch_caches[r].layers):
            for a, b in ((la.k_buf, lb.k_buf), (la.v_buf, lb.v_buf)):
                a, b = a[..., prefix:prefix + n, :].float(), b[..., prefix:prefix + n, :].float()
                assert ((a - b).abs().max() / a.abs().max()).item() <= TOL


def test_forward_batch_is_batch_invariant(cuda_device, model):
    """A request's logits do not depend on the other requests of its batch or their order."""
    from mdflash_b200.runner import Qwen3VerifyRunner
    dev = cuda_device
    runner = Qwen3VerifyRunner(model)
    trees, caches = [], []
    for r, (prefix, budget) in enumerate(REQUESTS):
        cache, tree = _request(runner, dev, prefix, budget, 40 + r)
        trees.append(tree)
        caches.append(cache)
    full = _batch(runner, dev, [0, 1, 2, 3], trees, caches)
    part = _batch(runner, dev, [3, 0], trees, caches)
    alone = _batch(runner, dev, [2], trees, caches)
    torch.cuda.synchronize()
    K.check_status(K.attention_status(dev))
    assert torch.equal(full[0], part[0]) and torch.equal(full[3], part[3])
    assert torch.equal(full[2], alone[2])
