"""GPU parity of the CUDA kernels against the CPU oracle and the golden vectors.

Integer / topology / index work must be bit-exact; attention is checked against an fp32
reference on the same bf16 inputs with max |err| / max |ref| <= 2e-2 (bf16 tolerance).
"""
import math

import numpy as np
import pytest
import torch

import inputs as gin
import oracle
from mdflash_b200 import kernels as K
from mdflash_b200._lib import DDTreeError
from parity_util import elem_rel_err

pytestmark = pytest.mark.gpu
ATTN_TOL = 2e-2


def _rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)).item()


# ----------------------------------------------------------------------------- tree
@pytest.mark.parametrize("spec", gin.TREE_CASES, ids=[c["name"] for c in gin.TREE_CASES])
def test_topk_tree_matches_reference(golden, cuda_device, spec):
    name = spec["name"]
    logits = gin.tree_logits(spec)
    budget = spec["budget"]
    root = torch.tensor([4242], dtype=torch.int64, device=cuda_device)
    tree = K.topk_tree(logits.to(cuda_device), budget, root_token=root, start=100)
    torch.cuda.synchronize()
    g_ids = golden[f"{name}/node_ids"]
    g_depths = golden[f"{name}/depths"]
    g_parents = golden[f"{name}/parents"]
    cnt = int(tree.node_count.item())
    assert cnt == g_ids.size == tree.n_nodes - 1
    np.testing.assert_array_equal(tree.node_token_ids[:cnt].cpu().numpy(), g_ids)
    np.testing.assert_array_equal(tree.node_depths[:cnt].cpu().numpy(), g_depths)
    np.testing.assert_array_equal(tree.parents[:cnt + 1].cpu().numpy(), g_parents)
    n = cnt + 1
    vis = np.unpackbits(golden[f"{name}/visibility"], axis=-1, count=n).astype(bool)
    bits = tree.anc_bits[:n].cpu().numpy().view(np.uint32)
    got = np.unpackbits(bits.view(np.uint8), axis=-1, bitorder="little", count=n).astype(bool)
    np.testing.assert_array_equal(got, vis)
    ids = tree.verify_ids[:n].cpu().numpy()
    pos = tree.verify_pos[:n].cpu().numpy()
    assert ids[0] == 4242 and pos[0] == 100
    np.testing.assert_array_equal(ids[1:], g_ids)
    np.testing.assert_array_equal(pos[1:], g_depths + 100)
    if budget > 0 and spec["L"] > 0:
        k = min(budget, spec["V"])
        o_lp, o_ids, _ = oracle.logz_topk(logits, k)
        np.testing.assert_array_equal(tree.top_token_ids.cpu().numpy(), o_ids)
        np.testing.assert_array_equal(tree.top_log_probs.cpu().numpy(), o_lp)


def test_topk_tree_repeated_launches_reuse_workspace(cuda_device):
    spec = gin.TREE_CASES[1]
    logits = gin.tree_logits(spec).to(cuda_device)
    first = K.topk_tree(logits, spec["budget"])
    p0 = first.parents.clone()
    for _ in range(5):
        t = K.topk_tree(logits, spec["budget"], out=first)
    torch.cuda.synchronize()
    assert torch.equal(t.parents, p0)


def test_topk_tree_strided_rows(cuda_device):
    spec = gin.TREE_CASES[3]
    logits = gin.tree_logits(spec)
    padded = torch.zeros((logits.shape[0], logits.shape[1] + 24), dtype=logits.dtype)
    padded[:, :logits.shape[1]] = logits
    view = padded.to(cuda_device)[:, :logits.shape[1]]
    tree = K.topk_tree(view, spec["budget"])
    ref = K.topk_tree(logits.to(cuda_device), spec["budget"])
    torch.cuda.synchronize()
    assert torch.equal(tree.parents, ref.parents)
    assert torch.equal(tree.node_token_ids, ref.node_token_ids)


# --------------------------------------------------------------------------- argmax
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,cols", [(33, 151936), (257, 151936), (5, 1001), (1, 7)])
def test_argmax_matches_oracle(cuda_device, dtype, rows, cols):
    g = torch.Generator().manual_seed(rows * 7 + cols)
    x = torch.randint(-4, 5, (rows, cols), generator=g).to(dtype)  # many exact ties
    got = K.argmax(x.to(cuda_device))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), oracle.argmax(x))
    np.testing.assert_array_equal(got.cpu().numpy(), torch.argmax(x.float(), -1).numpy())


def test_argmax_nan_and_strided(cuda_device):
    x = torch.randn(4, 1000)
    x[1, 17] = float("nan")
    x[1, 500] = float("nan")
    big = torch.zeros(4, 1024)
    big[:, :1000] = x
    got = K.argmax(big.to(cuda_device)[:, :1000])
    torch.cuda.synchronize()
    assert got.cpu().tolist() == oracle.argmax(x).tolist()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_argmax_signed_zero_ties_and_chunk_edges(cuda_device, dtype):
    """-0 and +0 are equal (lowest index wins); maxima placed on the edges of the per-CTA
    chunks, in the ragged tail, at both ends of the row; negative-only and NaN rows."""
    cols = 151936 + 5
    vec = 8 if dtype == torch.bfloat16 else 4       # elements per 16-byte load
    # edges of the per-CTA chunks for 4- and 8-way row splits, the ragged tail, both ends
    edges = sorted({c for parts in (4, 8) for j in (1, 2, 3)
                    for per in [-(-(cols // vec) // parts) * vec] for c in (j * per - 1, j * per)}
                   | {cols - 1, cols - 3, 0})
    x = torch.full((4 + len(edges), cols), -3.0)
    x[0, 100] = -0.0
    x[0, 90000] = 0.0                     # +0 after -0: the -0 index wins
    x[1, 5] = 0.0
    x[1, 7] = -0.0
    x[2] = -torch.arange(cols, dtype=torch.float32) - 1.0   # all negative, max at index 0
    x[3, 123] = float("nan")
    x[3, 77777] = float("inf")
    for r, c in enumerate(edges, start=4):
        x[r, c] = 2.0
    got = K.argmax(x.to(dtype).to(cuda_device))
    torch.cuda.synchronize()
    ref = oracle.argmax(x.to(dtype))
    np.testing.assert_array_equal(got.cpu().numpy(), ref)
    assert ref[0] == 100 and ref[1] == 5 and ref[2] == 0 and ref[3] == 123
    assert ref[4:].tolist() == edges


# ------------------------------------------------------------- accept walk + compaction
def _kv_cache(layers, heads, seq, dim, dtype, device, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn((1, heads, seq, dim), generator=g).to(dtype).to(device)
            for _ in range(2 * layers)]


@pytest.mark.parametrize("spec", gin.FOLLOW_CASES, ids=[c["name"] for c in gin.FOLLOW_CASES])
def test_accept_compact_matches_reference(golden, cuda_device, spec):
    tree_spec = next(c for c in gin.TREE_CASES if c["name"] == spec["tree"])
    tree = K.topk_tree(gin.tree_logits(tree_spec).to(cuda_device), tree_spec["budget"])
    n = tree.n_nodes
    post = torch.from_numpy(golden[f"{spec['name']}/posterior"]).to(cuda_device)
    past = 37
    cache = _kv_cache(3, 4, past + n + 5, 128, torch.bfloat16, cuda_device, 1)
    before = [t.cpu() for t in cache]
    kv = K.KvTable(cache)
    acc, n_acc, nxt = K.accept_compact(post, tree, kv, past)
    torch.cuda.synchronize()
    g_acc = golden[f"{spec['name']}/accepted"]
    cnt = int(n_acc.item())
    assert acc[:cnt].cpu().tolist() == g_acc.tolist()
    assert int(nxt.item()) == int(golden[f"{spec['name']}/next_token"][0])
    for t_after, t_before in zip(cache, before):
        ref = oracle.compact_rows(t_before.float().numpy().copy(), past, g_acc.tolist())
        got = t_after.cpu().float().numpy()[..., :past + cnt, :]
        np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("spec", gin.COMPACT_CASES, ids=[c["name"] for c in gin.COMPACT_CASES])
def test_compact_kv_matches_reference_cpp_extension(golden, cuda_device, spec):
    layers = gin.compact_cache(spec)
    # head_dim 8 fp32 rows are 32 bytes: a valid 16-byte-vector layout
    tensors = []
    for k, v in layers:
        tensors += [torch.from_numpy(k.copy()).to(cuda_device), torch.from_numpy(v.copy()).to(cuda_device)]
    kv = K.KvTable(tensors)
    keep = list(spec["keep"])
    if keep:
        K.compact_kv(torch.tensor(keep, device=cuda_device), kv, spec["past"])
    torch.cuda.synchronize()
    L = spec["past"] + len(keep) if keep else spec["past"]
    for li in range(len(layers)):
        np.testing.assert_array_equal(tensors[2 * li].cpu().numpy()[..., :L, :],
                                      golden[f"{spec['name']}/k{li}"])
        np.testing.assert_array_equal(tensors[2 * li + 1].cpu().numpy()[..., :L, :],
                                      golden[f"{spec['name']}/v{li}"])


def test_compaction_overlap_hazard_chain(cuda_device):
    """accepted = [0, 1, 2, 3, ...] shifted by one: row j reads j + 1 while row j + 1 is
    itself moved; staging the slice before any store keeps the reference semantics."""
    past, cur, dim = 5, 20, 128
    cache = _kv_cache(1, 2, past + cur, dim, torch.bfloat16, cuda_device, 3)
    before = [t.cpu().float().numpy().copy() for t in cache]
    keep = [0] + list(range(2, 17))
    K.compact_kv(torch.tensor(keep, device=cuda_device), K.KvTable(cache), past)
    torch.cuda.synchronize()
    for t, b in zip(cache, before):
        ref = oracle.compact_rows(b, past, keep)
        np.testing.assert_array_equal(t.cpu().float().numpy()[..., :past + len(keep), :], ref)


# --------------------------------------------------------------------------- attention
def _sdpa_ref(q, k, v, vis, past, causal=False):
    return oracle.tree_attention(q.float().cpu(), k.float().cpu(), v.float().cpu(), vis, past,
                                 causal=causal)


@pytest.mark.parametrize("spec", gin.ATTN_CASES, ids=[c["name"] for c in gin.ATTN_CASES])
@pytest.mark.parametrize("splits", [1, 2, 0])
def test_tree_attention_matches_reference(golden, cuda_device, spec, splits):
    q, k, v, parents = gin.attn_inputs(spec)
    bits = torch.from_numpy(oracle.ancestor_bits(parents).view(np.int32)).to(cuda_device)
    qd = q.transpose(0, 1).contiguous().to(torch.bfloat16).to(cuda_device)  # [N, Hq, D]
    out = K.tree_attention(qd, k.to(torch.bfloat16).to(cuda_device),
                           v.to(torch.bfloat16).to(cuda_device), bits, spec["past"],
                           kv_splits=splits)
    torch.cuda.synchronize()
    ref = torch.from_numpy(golden[f"{spec['name']}/out"])  # [N, Hq, D] from the reference
    assert _rel_err(out.cpu(), ref) <= ATTN_TOL


@pytest.mark.parametrize("hq,hkv,past,n,seed", [
    (32, 8, 4096, 65, 0),      # op-level tree attention shape (4k prefix, 64-node tree)
    (32, 8, 8192, 257, 1),     # Qwen3-8B verify shape, 256-node tree
    (16, 8, 512, 33, 2),       # Qwen3-0.6B-shaped verify
    (32, 8, 1000, 513, 3),     # prefix not a tile multiple, many tree tiles
    (8, 8, 300, 100, 4),       # no GQA sharing (group 1)
    (8, 8, 2048, 40, 5),       # 8 units x 17 key tiles over 136 CTAs: 16 parts per unit,
                               # merged in three batches
])
def test_tree_attention_shapes(cuda_device, hq, hkv, past, n, seed):
    g = torch.Generator().manual_seed(seed)
    d = 128
    sc = 1.0 / math.sqrt(d)
    q = (torch.randn((hq, n, d), generator=g) * sc).to(torch.bfloat16)
    k = (torch.randn((hkv, past + n, d), generator=g) * sc).to(torch.bfloat16)
    v = (torch.randn((hkv, past + n, d), generator=g) * sc).to(torch.bfloat16)
    parents = gin.random_tree(n, seed + 10)
    vis = oracle.visibility(parents)
    bits = torch.from_numpy(oracle.ancestor_bits(parents).view(np.int32)).to(cuda_device)
    out = K.tree_attention(q.transpose(0, 1).contiguous().to(cuda_device), k.to(cuda_device),
                           v.to(cuda_device), bits, past)
    torch.cuda.synchronize()
    ref = _sdpa_ref(q, k, v, vis, past)
    assert _rel_err(out.cpu(), ref) <= ATTN_TOL
    assert elem_rel_err(out.cpu(), ref) <= ATTN_TOL


def test_tree_attention_fp32_inputs(cuda_device):
    """An fp32 model's q / k / v: rounded to bf16 for the kernel, the output returned in
    fp32, within the bf16 tolerance of fp32 attention."""
    g = torch.Generator().manual_seed(21)
    hq, hkv, past, n, d = 16, 8, 512, 33, 128
    q = torch.randn((n, hq, d), generator=g) * 0.09
    k = torch.randn((hkv, past + n, d), generator=g) * 0.09
    v = torch.randn((hkv, past + n, d), generator=g)
    parents = gin.random_tree(n, 8)
    bits = torch.from_numpy(oracle.ancestor_bits(parents).view(np.int32)).to(cuda_device)
    out = K.tree_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), bits, past)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    ref = _sdpa_ref(q.transpose(0, 1), k, v, oracle.visibility(parents), past)
    assert _rel_err(out.cpu(), ref) <= ATTN_TOL
    assert elem_rel_err(out.cpu(), ref) <= ATTN_TOL


def test_tree_attention_wait_timeout_sets_status(cuda_device):
    """Every wait of the attention kernel is bounded.  ddt_tree_attn_wait_check launches the
    kernel with its load-issuing warp withholding every load, so the consumers' waits run out
    (after 2 ms here): the kernel must return, set the status word (read by check_status as
    DDT_ERR_TIMEOUT) and leave the context usable for the next launch."""
    g = torch.Generator().manual_seed(3)
    hq, hkv, past, n, d = 32, 8, 256, 65, 128
    q = (torch.randn((n, hq, d), generator=g) * 0.09).to(torch.bfloat16).to(cuda_device)
    k = (torch.randn((hkv, past + n, d), generator=g) * 0.09).to(torch.bfloat16).to(cuda_device)
    v = torch.randn((hkv, past + n, d), generator=g).to(torch.bfloat16).to(cuda_device)
    parents = gin.random_tree(n, 9)
    bits = torch.from_numpy(oracle.ancestor_bits(parents).view(np.int32)).to(cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    K.tree_attention_wait_check(q, k, v, bits, past, 2_000_000, status)
    torch.cuda.synchronize()
    assert int(status.item()) != 0
    with pytest.raises(DDTreeError, match="bounded device wait expired"):
        K.check_status(status)
    assert int(status.item()) == 0
    # the same sizes right after, on the same status word: correct and no timeout
    out = K.tree_attention(q, k, v, bits, past, status=status)
    torch.cuda.synchronize()
    K.check_status(status)
    ref = _sdpa_ref(q.transpose(0, 1), k, v, oracle.visibility(parents), past)
    assert _rel_err(out.cpu(), ref) <= ATTN_TOL


@pytest.mark.parametrize("hq,hkv,ctx,n", [(32, 8, 700, 16), (16, 8, 0, 16), (32, 8, 4000, 64)])
def test_tree_attention_unmasked_drafter_attention(cuda_device, hq, hkv, ctx, n):
    """The DFlash drafter's attention (model/dflash.py:58-102): a block of n noise queries
    over context + block keys, non-causal, no mask; through the kernel's unmasked mode and
    through the plug-in on a module with is_causal = False."""
    from mdflash_b200 import attention as A
    g = torch.Generator().manual_seed(ctx + n)
    d = 128
    q = (torch.randn((1, hq, n, d), generator=g) * 0.09).to(torch.bfloat16)
    k = (torch.randn((1, hkv, ctx + n, d), generator=g) * 0.09).to(torch.bfloat16)
    v = torch.randn((1, hkv, ctx + n, d), generator=g).to(torch.bfloat16)
    ref = oracle.tree_attention(q[0], k[0], v[0], np.ones((n, n), bool), ctx)
    out = K.tree_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, ctx,
                           unmasked=True)

    class _Drafter(torch.nn.Module):
        is_causal = False

    plug, _ = A.ddtree_attention_forward(_Drafter(), q.to(cuda_device), k.to(cuda_device),
                                         v.to(cuda_device), None, scaling=d ** -0.5)
    torch.cuda.synchronize()
    for o in (out.cpu(), plug[0].cpu()):
        assert _rel_err(o, ref) <= ATTN_TOL
        assert elem_rel_err(o, ref) <= ATTN_TOL


def test_tree_attention_hf_layout_and_causal(cuda_device):
    """HF passes query as a [1, Hq, N, D] view of [1, N, Hq, D]; prefill is causal."""
    g = torch.Generator().manual_seed(9)
    hq, hkv, n, past, d = 16, 8, 300, 0, 128
    q_nhd = (torch.randn((1, n, hq, d), generator=g) * 0.1).to(torch.bfloat16).to(cuda_device)
    q = q_nhd.transpose(1, 2)
    k = (torch.randn((1, hkv, n, d), generator=g) * 0.1).to(torch.bfloat16).to(cuda_device)
    v = torch.randn((1, hkv, n, d), generator=g).to(torch.bfloat16).to(cuda_device)
    out = K.tree_attention(q, k, v, None, past, causal=True)
    torch.cuda.synchronize()
    ref = _sdpa_ref(q[0].cpu(), k[0].cpu(), v[0].cpu(), None, past, causal=True)
    assert _rel_err(out.cpu(), ref) <= ATTN_TOL


def test_tree_attention_partial_merge_equals_full(cuda_device):
    """Split the key range in 3 shards, compute partials, merge: equals the full call."""
    g = torch.Generator().manual_seed(5)
    hq, hkv, past, n, d = 32, 8, 3000, 129, 128
    q = (torch.randn((n, hq, d), generator=g) * 0.09).to(torch.bfloat16).to(cuda_device)
    k = (torch.randn((hkv, past + n, d), generator=g) * 0.09).to(torch.bfloat16).to(cuda_device)
    v = torch.randn((hkv, past + n, d), generator=g).to(torch.bfloat16).to(cuda_device)
    parents = gin.random_tree(n, 77)
    bits = torch.from_numpy(oracle.ancestor_bits(parents).view(np.int32)).to(cuda_device)
    full = K.tree_attention(q, k, v, bits, past, kv_splits=1)
    bounds = [0, 1100, 2600, past + n]
    parts = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        parts.append(K.tree_attention_partial(q, k[:, a:b], v[:, a:b], a, b, bits, past))
    o = torch.cat([p[0] for p in parts])  # each shard: [S, rows, D] partials
    m = torch.cat([p[1] for p in parts])
    l = torch.cat([p[2] for p in parts])
    merged = K.attn_merge(o, m, l, n, hq)
    torch.cuda.synchronize()
    assert _rel_err(merged, full) <= 1e-2


def test_mask_to_bits_roundtrip(cuda_device):
    parents = gin.random_tree(200, 4)
    vis = oracle.visibility(parents)
    mask = torch.zeros((200, 200), dtype=torch.bfloat16)
    mask.masked_fill_(~torch.from_numpy(vis), torch.finfo(torch.bfloat16).min)
    bits = K.mask_to_bits(mask.to(cuda_device))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32),
                                  oracle.ancestor_bits(parents))


def test_gather_rows_device_count(cuda_device):
    """ddt_gather_rows: rows idx[i] for i < the device count, out-of-range indices give zero
    rows, rows past the count keep their contents."""
    g = torch.Generator(device=cuda_device).manual_seed(4)
    src = torch.randn((40, 3, 64), generator=g, device=cuda_device).to(torch.bfloat16)
    idx = torch.tensor([5, 0, 39, 7, 40, -1, 2], dtype=torch.int64, device=cuda_device)
    out = torch.full((7, 3, 64), 9.0, dtype=torch.bfloat16, device=cuda_device)
    count = torch.tensor([6], dtype=torch.int32, device=cuda_device)
    K.gather_rows(src, idx, count=count, out=out)
    torch.cuda.synchronize()
    for i, j in enumerate([5, 0, 39, 7]):
        assert torch.equal(out[i], src[j])
    assert bool((out[4] == 0).all()) and bool((out[5] == 0).all())
    assert bool((out[6] == 9.0).all())
    full = K.gather_rows(src, idx[:4])
    torch.cuda.synchronize()
    assert torch.equal(full, src[idx[:4]])
