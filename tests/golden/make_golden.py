"""Generate the golden fixtures in tests/golden/ by running the reference's own code.

Run where the DDTree research code is checked out: --reference PATH, or the environment
variable DDTREE_REFERENCE.  It imports ddtree.py / dflash.py / model/ unchanged except:
  * ``cuda_time`` is replaced by ``time.perf_counter`` (the original calls
    torch.cuda.synchronize, dflash.py:140-142, and this generator runs on a CPU);
  * for inputs with value ties (bf16 logits, crafted small vocabularies) ``torch.topk``
    inside ddtree is wrapped with a stable selection, value descending then index
    ascending, because torch.topk leaves the order of equal values unspecified.

Inputs are regenerated from numpy seeds by tests/golden/inputs.py, so only seeds and
outputs are stored.  The fixtures are small .npz files.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs as gin  # noqa: E402


def load_reference(path: str):
    sys.path.insert(0, path)
    import dflash  # noqa: F401
    dflash.cuda_time = time.perf_counter
    import ddtree
    ddtree.cuda_time = time.perf_counter
    return ddtree


class StableTopk:
    """torch.topk replacement with (value desc, index asc) order on ties."""

    def __init__(self, orig):
        self.orig = orig

    def __call__(self, x, k, dim=-1, largest=True, sorted=True):
        assert largest and dim in (-1, x.dim() - 1)
        n = x.shape[-1]
        idx = torch.arange(n, dtype=torch.long).expand_as(x)
        # sort by value desc, then index asc: stable sort on -value keeps index order
        order = torch.sort(-x, dim=-1, stable=True).indices
        top_ids = order[..., :k]
        return torch.gather(x, -1, top_ids), top_ids


def ref_top(ddtree, logits: torch.Tensor, k: int):
    """The exact tensor ops of ddtree.py:106-109."""
    lf = logits.float()
    top, ids = ddtree.torch.topk(lf, k=k, dim=-1)
    lz = torch.logsumexp(lf, dim=-1, keepdim=True)
    return (top - lz).to(torch.float32), ids.to(torch.long), lz[:, 0]


def gen_trees(ddtree, out: dict, manifest: dict):
    cases = []
    for spec in gin.TREE_CASES:
        logits = gin.tree_logits(spec)
        budget = spec["budget"]
        stable = spec["stable"]
        orig = ddtree.torch.topk
        if stable:
            ddtree.torch.topk = StableTopk(orig)
        try:
            res = ddtree.build_ddtree_tree(logits, budget)
            if budget > 0 and logits.shape[0] > 0:
                k = min(budget, logits.shape[-1])
                top_lp, top_ids, lz = ref_top(ddtree, logits, k)
            else:
                top_lp = torch.zeros((0, 0)); top_ids = torch.zeros((0, 0), dtype=torch.long)
                lz = torch.zeros((0,))
        finally:
            ddtree.torch.topk = orig
        if not stable and budget > 0 and logits.shape[0] > 0:
            # fp32 inputs: the unmodified reference must agree with the stable order
            ddtree.torch.topk = StableTopk(orig)
            try:
                res_s = ddtree.build_ddtree_tree(logits, budget)
            finally:
                ddtree.torch.topk = orig
            assert res_s[2] == res[2] and torch.equal(res_s[0], res[0]), spec
        node_ids, depths, parents, child_maps, vis, _ = res
        name = spec["name"]
        out[f"{name}/node_ids"] = node_ids.numpy().astype(np.int64)
        out[f"{name}/depths"] = depths.numpy().astype(np.int64)
        out[f"{name}/parents"] = np.asarray(parents, np.int32)
        out[f"{name}/visibility"] = np.packbits(vis.numpy().astype(np.uint8), axis=-1)
        out[f"{name}/top_lp"] = top_lp.numpy()
        out[f"{name}/top_ids"] = top_ids.numpy()
        out[f"{name}/logz"] = lz.numpy().astype(np.float32)
        cases.append(name)
    manifest["trees"] = cases


def gen_compile(ddtree, out: dict, manifest: dict):
    cases = []
    for spec in gin.COMPILE_CASES:
        tree_name = spec["tree"]
        node_ids = torch.from_numpy(out[f"{tree_name}/node_ids"])
        depths = torch.from_numpy(out[f"{tree_name}/depths"])
        parents = out[f"{tree_name}/parents"]
        n = parents.shape[0]
        vis = torch.from_numpy(np.unpackbits(out[f"{tree_name}/visibility"], axis=-1,
                                             count=n).astype(bool))
        past, prev_start, prev_len = spec["past"], spec["prev_start"], spec["prev_len"]
        cap = spec["cap"]
        dtype = getattr(torch, spec["dtype"])
        ids_buf = torch.full((1, cap), -7, dtype=torch.long)
        pos_buf = torch.full((1, cap), -7, dtype=torch.long)
        mask_buf = torch.zeros((1, 1, cap, past + cap + 8), dtype=dtype)
        if prev_len > 0:
            mask_buf[0, 0, :prev_len, prev_start:prev_start + prev_len] = torch.finfo(dtype).min
        vis_buf = torch.zeros((cap, cap), dtype=torch.bool)
        ids, pos, mask, pl, cl = ddtree.compile_ddtree_tree(
            torch.tensor(spec["root"]), spec["start"], node_ids, depths, vis, past, dtype,
            torch.device("cpu"), ids_buf, pos_buf, mask_buf, vis_buf, prev_start, prev_len)
        name = spec["name"]
        out[f"{name}/ids"] = ids.numpy().copy()
        out[f"{name}/pos"] = pos.numpy().copy()
        out[f"{name}/mask"] = mask.float().numpy().copy()
        out[f"{name}/mask_buffer"] = mask_buf.float().numpy().copy()
        out[f"{name}/lengths"] = np.array([pl, cl], np.int64)
        cases.append(name)
    manifest["compile"] = cases


def gen_follow(ddtree, out: dict, manifest: dict):
    cases = []
    for spec in gin.FOLLOW_CASES:
        tree_name = spec["tree"]
        node_ids = out[f"{tree_name}/node_ids"]
        parents = out[f"{tree_name}/parents"]
        child_maps = [dict() for _ in range(parents.shape[0])]
        for i in range(1, parents.shape[0]):
            child_maps[int(parents[i])][int(node_ids[i - 1])] = i
        post = gin.follow_posterior(spec, node_ids, parents)
        acc, nxt = ddtree.follow_verified_tree(child_maps, torch.from_numpy(post)[None])
        name = spec["name"]
        out[f"{name}/posterior"] = post
        out[f"{name}/accepted"] = np.asarray(acc, np.int64)
        out[f"{name}/next_token"] = np.asarray([nxt], np.int64)
        cases.append(name)
    manifest["follow"] = cases


def gen_compact(ddtree, out: dict, manifest: dict, use_cpp: bool):
    from transformers import DynamicCache
    cases = []
    if use_cpp:
        ddtree.maybe_enable_cpp_compact(True)
        assert ddtree.load_cpp_compact_module() is not None
    for spec in gin.COMPACT_CASES:
        layers = gin.compact_cache(spec)
        cache = DynamicCache()
        for li, (k, v) in enumerate(layers):
            cache.update(torch.from_numpy(k.copy()), torch.from_numpy(v.copy()), li)
        ddtree.compact_dynamic_cache(cache, spec["past"], list(spec["keep"]))
        name = spec["name"]
        for li, layer in enumerate(cache.layers):
            out[f"{name}/k{li}"] = layer.keys.numpy().copy()
            out[f"{name}/v{li}"] = layer.values.numpy().copy()
        out[f"{name}/seq_len"] = np.array([cache.get_seq_length()], np.int64)
        cases.append(name)
    manifest["compact"] = cases
    manifest["compact_cpp"] = bool(use_cpp)


def gen_attention(ddtree, out: dict, manifest: dict):
    """Reference verify attention: the mask from compile_ddtree_tree and the call
    transformers' sdpa_attention_forward makes (enable_gqa, scale=D^-1/2)."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    cases = []
    for spec in gin.ATTN_CASES:
        q, k, v, parents = gin.attn_inputs(spec)
        n = parents.shape[0]
        past = spec["past"]
        vis = np.zeros((n, n), bool)
        vis[0, 0] = True
        for i in range(1, n):
            vis[i, :i] = vis[parents[i], :i]
            vis[i, i] = True
        dtype = torch.float32
        mask_buf = torch.zeros((1, 1, n, past + n), dtype=dtype)
        block = mask_buf[0, 0, :n, past:past + n]
        block.fill_(torch.finfo(dtype).min)
        block.masked_fill_(torch.from_numpy(vis), 0)

        class _M(torch.nn.Module):
            num_key_value_groups = q.shape[0] // k.shape[0]
            is_causal = True

        o, _ = sdpa_attention_forward(_M(), q[None].float(), k[None].float(), v[None].float(),
                                      mask_buf, scaling=q.shape[-1] ** -0.5)
        name = spec["name"]
        out[f"{name}/out"] = o[0].numpy().copy()
        out[f"{name}/parents"] = parents
        cases.append(name)
    manifest["attention"] = cases


def gen_sampled(ddtree, out: dict, manifest: dict, reference: str):
    """build_sampled_candidate_tree on seeded chains, and sample_candidate_chains at
    temperature 0 on seeded logits."""
    cases = []
    for spec in gin.SAMPLED_CASES:
        chains = gin.sampled_chains(spec)
        node_ids, depths, parents, child_maps, vis = ddtree.build_sampled_candidate_tree(
            chains, spec["budget"])
        name = spec["name"]
        out[f"{name}/node_ids"] = node_ids.numpy().astype(np.int64)
        out[f"{name}/depths"] = depths.numpy().astype(np.int64)
        out[f"{name}/parents"] = np.asarray(parents, np.int32)
        out[f"{name}/visibility"] = np.packbits(vis.numpy(), axis=-1)
        cases.append(name)
    manifest["sampled"] = cases
    import mdflash  # noqa: F401  (the reference's module; imports ddtree / dflash / model)
    spec = gin.GREEDY_CHAIN_CASE
    logits = gin._logits(spec["seed"], spec["L"], spec["V"], "normal3")
    chains = mdflash.sample_candidate_chains(torch.from_numpy(logits), spec["S"], 0.0)
    out["greedy_chains/chains"] = chains.numpy().astype(np.int64)
    manifest["greedy_chains"] = dict(spec)


def gen_loop(ddtree, out: dict, manifest: dict):
    """The reference's own decode loop, ddtree_generate (ddtree.py:338-530), for a few rounds
    on the tiny fp32 target with the stub drafter: output ids and per-round acceptance."""
    spec = gin.LOOP_CASE
    target = gin.loop_target(spec)
    drafter = gin.StubDrafter(spec["hidden"])
    ids = gin.loop_inputs(spec)
    res = ddtree.ddtree_generate(drafter, target, ids, spec["mask_token_id"],
                                 spec["max_new_tokens"], spec["block_size"], None, 0.0,
                                 spec["budget"])
    out["loop/output_ids"] = res.output_ids.numpy().astype(np.int64)
    out["loop/acceptance_lengths"] = np.asarray(res.acceptance_lengths, np.int64)
    manifest["loop"] = dict(spec)
    print("loop acceptance", res.acceptance_lengths)


def gen_e2e(ddtree, out: dict, manifest: dict):
    """One DDTree verify step on the CPU-runnable Qwen3-0.6B-shaped target (fp32)."""
    from transformers import DynamicCache
    spec = gin.E2E_CASE
    model = gin.e2e_model(spec)
    ids, draft_logits = gin.e2e_inputs(spec)
    P = ids.shape[1]
    B = spec["budget"]
    N = B + 1
    with torch.inference_mode():
        cache = DynamicCache()
        o = model(ids, position_ids=torch.arange(P)[None], past_key_values=cache, use_cache=True,
                  logits_to_keep=1)
        root = o.logits.argmax(-1)[0, -1]
        root_top2 = torch.topk(o.logits[0, -1], 2)
        res = ddtree.build_ddtree_tree(draft_logits, B)
        node_ids, depths, parents, child_maps, vis, _ = res
        ids_buf = torch.empty((1, N), dtype=torch.long)
        pos_buf = torch.empty((1, N), dtype=torch.long)
        mask_buf = torch.zeros((1, 1, N, P + N), dtype=torch.float32)
        vis_buf = torch.empty((N, N), dtype=torch.bool)
        vi, vp, am, _, _ = ddtree.compile_ddtree_tree(root, P, node_ids, depths, vis, P,
                                                      torch.float32, torch.device("cpu"), ids_buf,
                                                      pos_buf, mask_buf, vis_buf, 0, 0)
        o2 = model(vi, position_ids=vp, attention_mask=am, past_key_values=cache, use_cache=True)
        logits = o2.logits[0]
        post = logits.argmax(-1)
        acc, nxt = ddtree.follow_verified_tree(child_maps, post[None])
        top2v, top2i = torch.topk(logits, 2, dim=-1)
        top2 = top2v
        kv_before = [(l.keys.clone(), l.values.clone()) for l in cache.layers]
        ddtree.compact_dynamic_cache(cache, P, acc)
    out["e2e/root"] = np.array([int(root)], np.int64)
    out["e2e/node_ids"] = node_ids.numpy()
    out["e2e/depths"] = depths.numpy()
    out["e2e/parents"] = np.asarray(parents, np.int32)
    out["e2e/posterior"] = post.numpy().astype(np.int64)
    out["e2e/logit_top2"] = top2.numpy()
    out["e2e/logits_row_sum"] = logits.double().sum(-1).numpy()
    out["e2e/logit_top2_ids"] = top2i.numpy().astype(np.int64)
    out["e2e/root_top2"] = root_top2.values.numpy()
    out["e2e/root_top2_ids"] = root_top2.indices.numpy().astype(np.int64)
    # a seeded sample of 4096 vocabulary columns of every verify row, for per-element checks
    cols = np.sort(np.random.default_rng(20260).choice(logits.shape[-1], 4096, replace=False))
    out["e2e/logit_cols"] = cols.astype(np.int64)
    out["e2e/logit_sample"] = logits[:, torch.from_numpy(cols)].numpy().astype(np.float32)
    out["e2e/accepted"] = np.asarray(acc, np.int64)
    out["e2e/next_token"] = np.array([nxt], np.int64)
    out["e2e/seq_len_after"] = np.array([cache.get_seq_length()], np.int64)
    # layer-0 keys of the tree window before compaction (small) to pin the verify K/V
    out["e2e/k0_tree"] = kv_before[0][0][0, :, P:, :].numpy().copy()
    manifest["e2e"] = dict(spec)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DDTREE_REFERENCE"),
                    help="checkout of the DDTree research code (default: $DDTREE_REFERENCE)")
    ap.add_argument("--only", default="",
                    help="comma-separated groups to regenerate (e2e, sampled, loop), keeping the other "
                         "arrays of golden.npz")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--no-cpp", action="store_true")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference PATH (or DDTREE_REFERENCE) is required")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    # the reference builds its inline C++ extension; keep that build out of the home dir
    os.environ.setdefault("TORCH_EXTENSIONS_DIR", tempfile.mkdtemp(prefix="ddtree_ref_ext_"))
    ddtree = load_reference(args.reference)
    out: dict = {}
    manifest: dict = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__}
    t0 = time.time()
    if args.only:
        groups = set(args.only.split(","))
        prefixes = {"e2e": ("e2e/",),
                    "sampled": tuple(f"{c['name']}/" for c in gin.SAMPLED_CASES) +
                    ("greedy_chains/",),
                    "loop": ("loop/",)}
        drop = tuple(p for g in groups for p in prefixes[g])
        old = np.load(os.path.join(HERE, "golden.npz"))
        out = {k: old[k] for k in old.files if not k.startswith(drop)}
        with open(os.path.join(HERE, "manifest.json")) as f:
            manifest = json.load(f)
        if "e2e" in groups:
            gen_e2e(ddtree, out, manifest)
        if "sampled" in groups:
            gen_sampled(ddtree, out, manifest, args.reference)
        if "loop" in groups:
            gen_loop(ddtree, out, manifest)
        np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
        with open(os.path.join(HERE, "manifest.json"), "w") as f:
            json.dump(manifest, f, indent=1, sort_keys=True)
        print(f"wrote {len(out)} arrays in {time.time() - t0:.1f}s")
        return
    gen_trees(ddtree, out, manifest)
    gen_compile(ddtree, out, manifest)
    gen_follow(ddtree, out, manifest)
    gen_compact(ddtree, out, manifest, use_cpp=not args.no_cpp)
    gen_attention(ddtree, out, manifest)
    gen_sampled(ddtree, out, manifest, args.reference)
    gen_loop(ddtree, out, manifest)
    if not args.skip_e2e:
        gen_e2e(ddtree, out, manifest)
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print(f"wrote {len(out)} arrays in {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
