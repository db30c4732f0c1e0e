"""Seeded input generators shared by make_golden.py and the tests.

Every input of a golden case is regenerated here from a numpy seed (PCG64), so the
fixtures only hold outputs, and the GPU tests can rebuild the exact inputs without
the reference code.
"""
from __future__ import annotations

import numpy as np
import torch

V_QWEN3 = 151936


def _logits(seed: int, L: int, V: int, kind: str) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind == "normal3":
        return rng.standard_normal((L, V)).astype(np.float32) * np.float32(3.0)
    if kind == "ties":  # three distinct values: massive ties everywhere
        return rng.integers(0, 3, (L, V)).astype(np.float32) * np.float32(0.5)
    if kind == "spiky":  # one dominant logit per row: log-probs of exactly 0 appear
        x = rng.standard_normal((L, V)).astype(np.float32)
        x[np.arange(L), rng.integers(0, V, L)] = np.float32(200.0)
        return x
    raise ValueError(kind)


def _case(name, seed, L, V, budget, dtype, kind="normal3"):
    return dict(name=name, seed=seed, L=L, V=V, budget=budget, dtype=dtype, kind=kind,
                stable=(dtype != "float32" or kind != "normal3"))


TREE_CASES = [
    _case("fp32_b32_s0", 0, 15, V_QWEN3, 32, "float32"),
    _case("fp32_b256_s1", 1, 15, V_QWEN3, 256, "float32"),
    _case("fp32_b512_s2", 2, 15, V_QWEN3, 512, "float32"),
    _case("bf16_b64_s3", 3, 15, V_QWEN3, 64, "bfloat16"),
    _case("bf16_b256_s4", 4, 15, V_QWEN3, 256, "bfloat16"),
    _case("bf16_b512_s5", 5, 15, V_QWEN3, 512, "bfloat16"),
    _case("bf16_b1024_s6", 6, 15, V_QWEN3, 1024, "bfloat16"),
    _case("ties_v50_b10", 7, 4, 50, 10, "float32", "ties"),
    _case("ties_v50_b200", 8, 4, 50, 200, "float32", "ties"),
    _case("ties_bf16_v4000_b300", 9, 6, 4000, 300, "bfloat16", "ties"),
    _case("tiny_v3_l3_b40", 10, 3, 3, 40, "float32"),
    _case("spiky_v1000_b20", 11, 5, 1000, 20, "float32", "spiky"),
    _case("one_b1", 12, 15, 1000, 1, "float32"),
    _case("depth1_b8", 13, 1, 1000, 8, "float32"),
    _case("empty_b0", 14, 15, 1000, 0, "float32"),
    _case("empty_l0", 15, 0, 1000, 8, "float32"),
]


def tree_logits(spec: dict) -> torch.Tensor:
    x = torch.from_numpy(_logits(spec["seed"], spec["L"], spec["V"], spec["kind"]))
    return x.to(getattr(torch, spec["dtype"]))


COMPILE_CASES = [
    dict(name="compile_bf16", tree="ties_v50_b10", root=7, start=20, past=20, cap=14,
         prev_start=5, prev_len=4, dtype="bfloat16"),
    dict(name="compile_fp32", tree="spiky_v1000_b20", root=3, start=33, past=33, cap=25,
         prev_start=0, prev_len=0, dtype="float32"),
]


def _children(parents: np.ndarray) -> list[list[int]]:
    ch: list[list[int]] = [[] for _ in range(parents.shape[0])]
    for i in range(1, parents.shape[0]):
        ch[int(parents[i])].append(i)
    return ch


def follow_posterior(spec: dict, node_ids: np.ndarray, parents: np.ndarray) -> np.ndarray:
    """Posterior tokens [N] for the accept walk.  kind:
      random  - uniform tokens (almost always accepts only the root)
      path    - follows the root->target path, then a token that is not a child
      none    - the root's token is not a child of the root
    """
    rng = np.random.default_rng(spec["seed"])
    n = parents.shape[0]
    V = spec["V"]
    post = rng.integers(0, V, n).astype(np.int64)
    ch = _children(parents)
    tok = lambda i: int(node_ids[i - 1])  # noqa: E731
    if spec["kind"] == "random":
        return post
    if spec["kind"] == "none":
        used = {tok(c) for c in ch[0]}
        t = 0
        while t in used:
            t += 1
        post[0] = t
        return post
    if spec["kind"] == "path":
        target = spec["target"]
        if target < 0:  # deepest node, lowest index among the deepest
            depth = np.zeros(n, np.int64)
            for i in range(1, n):
                depth[i] = depth[parents[i]] + 1
            target = int(np.argmax(depth))
        path = [target]
        while path[-1] != 0:
            path.append(int(parents[path[-1]]))
        path = path[::-1]
        for a, b in zip(path[:-1], path[1:]):
            post[a] = tok(b)
        used = {tok(c) for c in ch[target]}
        t = int(post[target])
        while t in used:
            t = (t + 1) % V
        post[target] = t
        return post
    raise ValueError(spec["kind"])


FOLLOW_CASES = [
    dict(name="follow_random", tree="fp32_b256_s1", kind="random", seed=100, V=V_QWEN3),
    dict(name="follow_none", tree="fp32_b256_s1", kind="none", seed=101, V=V_QWEN3),
    dict(name="follow_deepest", tree="fp32_b256_s1", kind="path", target=-1, seed=102,
         V=V_QWEN3),
    dict(name="follow_node40", tree="bf16_b256_s4", kind="path", target=40, seed=103,
         V=V_QWEN3),
    dict(name="follow_deepest_b1024", tree="bf16_b1024_s6", kind="path", target=-1, seed=104,
         V=V_QWEN3),
    dict(name="follow_ties", tree="ties_v50_b200", kind="path", target=-1, seed=105, V=50),
]


COMPACT_CASES = [
    dict(name=f"compact_{tag}", seed=200 + i, layers=2, heads=2, past=10, cur=9, dim=8,
         keep=keep)
    for i, (tag, keep) in enumerate([
        ("root", [0]),
        ("sparse", [0, 2, 5]),
        ("identity", [0, 1, 2]),
        ("all", list(range(9))),
        ("empty", []),
        ("tail", [0, 1, 4, 8]),
        ("chain", [0, 3, 4, 6, 7, 8]),
    ])
]


def compact_cache(spec: dict) -> list[tuple[np.ndarray, np.ndarray]]:
    rng = np.random.default_rng(spec["seed"])
    S = spec["past"] + spec["cur"]
    shape = (1, spec["heads"], S, spec["dim"])
    return [(rng.standard_normal(shape).astype(np.float32),
             rng.standard_normal(shape).astype(np.float32)) for _ in range(spec["layers"])]


def random_tree(n: int, seed: int, max_depth: int = 16, p: float = 0.5) -> np.ndarray:
    """Parents of a seeded random tree with n nodes (root included): BFS growth, child
    counts ~ Geometric(p) on {0, 1, ...}, depth <= max_depth.  If growth stops early the
    next node attaches to the lowest-index node that may still have children."""
    rng = np.random.default_rng(seed)
    parents = [-1]
    depth = [0]
    queue = [0]
    qi = 0
    while len(parents) < n:
        if qi == len(queue):
            cand = next(i for i in range(len(parents)) if depth[i] < max_depth)
            queue.append(cand)
        node = queue[qi]
        qi += 1
        if depth[node] >= max_depth:
            continue
        c = int(rng.geometric(p)) - 1
        for _ in range(c):
            if len(parents) >= n:
                break
            parents.append(node)
            depth.append(depth[node] + 1)
            queue.append(len(parents) - 1)
    return np.asarray(parents, np.int32)


ATTN_CASES = [
    dict(name="attn_h4_p37_n13", seed=300, hq=4, hkv=2, dim=128, past=37, n=13),
    dict(name="attn_h8_p200_n65", seed=301, hq=8, hkv=2, dim=128, past=200, n=65),
    dict(name="attn_h4_p0_n20", seed=302, hq=4, hkv=1, dim=128, past=0, n=20),
]


def bf16_exact(x: np.ndarray) -> torch.Tensor:
    """float32 tensor whose values are exactly representable in bf16."""
    return torch.from_numpy(x).to(torch.bfloat16).float()


def attn_inputs(spec: dict):
    """q [Hq, N, D], k/v [Hkv, past+N, D] (bf16-exact float32), parents [N]."""
    rng = np.random.default_rng(spec["seed"])
    d = spec["dim"]
    s = spec["past"] + spec["n"]
    sc = np.float32(1.0 / np.sqrt(d))
    q = bf16_exact(rng.standard_normal((spec["hq"], spec["n"], d)).astype(np.float32) * sc)
    k = bf16_exact(rng.standard_normal((spec["hkv"], s, d)).astype(np.float32) * sc)
    v = bf16_exact(rng.standard_normal((spec["hkv"], s, d)).astype(np.float32) * sc)
    parents = random_tree(spec["n"], spec["seed"] + 1)
    return q, k, v, parents


E2E_CASE = dict(name="qwen3_0p6b_shape_p512_b32", layers=28, hidden=1024, heads=16, kv_heads=8,
                head_dim=128, mlp=3072, vocab=V_QWEN3, rope_theta=1e6, prompt=512, depths=15,
                budget=32, model_seed=0, input_seed=0)


def qwen3_config(spec: dict, attn_implementation: str = "sdpa"):
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=spec["vocab"], hidden_size=spec["hidden"],
                       intermediate_size=spec["mlp"], num_hidden_layers=spec["layers"],
                       num_attention_heads=spec["heads"], num_key_value_heads=spec["kv_heads"],
                       head_dim=spec["head_dim"], rope_theta=spec["rope_theta"],
                       max_position_embeddings=40960, tie_word_embeddings=True,
                       attn_implementation=attn_implementation)


def e2e_model(spec: dict, attn_implementation: str = "sdpa"):
    from transformers import Qwen3ForCausalLM
    torch.manual_seed(spec["model_seed"])
    return Qwen3ForCausalLM(qwen3_config(spec, attn_implementation)).eval()


def e2e_inputs(spec: dict):
    rng = np.random.default_rng(spec["input_seed"])
    ids = torch.from_numpy(rng.integers(0, spec["vocab"], (1, spec["prompt"])).astype(np.int64))
    logits = torch.from_numpy(
        rng.standard_normal((spec["depths"], spec["vocab"])).astype(np.float32) * np.float32(3.0))
    return ids, logits


# Sampled-chain trees (build_sampled_candidate_tree, ddtree.py:169-224): chains over a small
# vocabulary so that prefixes are shared, budgets that cut a chain in the middle, exact fits,
# identical chains and the empty cases.
SAMPLED_CASES = [
    dict(name="chains_s32_l15_v4_b32", seed=400, S=32, L=15, V=4, budget=32),
    dict(name="chains_s256_l15_v3_b256", seed=401, S=256, L=15, V=3, budget=256),
    dict(name="chains_s1024_l15_v2_b1024", seed=402, S=1024, L=15, V=2, budget=1024),
    dict(name="chains_s512_l16_v6_b300", seed=403, S=512, L=16, V=6, budget=300),
    dict(name="chains_s20_l5_v50_b200", seed=404, S=20, L=5, V=50, budget=200),
    dict(name="chains_s64_l10_same_b64", seed=405, S=64, L=10, V=1, budget=64),
    dict(name="chains_s8_l20_v151936_b8", seed=406, S=8, L=20, V=151936, budget=8),
    dict(name="chains_s0_l15_b8", seed=407, S=0, L=15, V=4, budget=8),
    dict(name="chains_s8_l0_b8", seed=408, S=8, L=0, V=4, budget=8),
    dict(name="chains_s8_l4_b0", seed=409, S=8, L=4, V=4, budget=0),
]


def sampled_chains(spec: dict) -> torch.Tensor:
    rng = np.random.default_rng(spec["seed"])
    return torch.from_numpy(rng.integers(0, spec["V"], (spec["S"], spec["L"])).astype(np.int64))


# sample_candidate_chains at temperature 0 (mdflash.py:19-40): the argmax chain repeated
GREEDY_CHAIN_CASE = dict(name="greedy_chains", seed=410, L=15, V=V_QWEN3, S=16)


# A few rounds of ddtree_generate (ddtree.py:338-530) on a tiny fp32 target with a
# deterministic stand-in for the DFlash drafter.  The vocabulary is small (16) so that the
# tree's depth-1 candidates often hold the target's greedy token and rounds accept several
# tokens; the weights are large (initializer_range 0.2) so that greedy choices have wide
# margins.
LOOP_CASE = dict(name="loop_tiny", layers=2, hidden=256, heads=4, kv_heads=2, head_dim=128,
                 mlp=512, vocab=16, rope_theta=1e6, prompt=24, block_size=8, budget=64,
                 max_new_tokens=40, model_seed=3, input_seed=4, mask_token_id=15)


def loop_target(spec: dict):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=spec["vocab"], hidden_size=spec["hidden"],
                      intermediate_size=spec["mlp"], num_hidden_layers=spec["layers"],
                      num_attention_heads=spec["heads"], num_key_value_heads=spec["kv_heads"],
                      head_dim=spec["head_dim"], rope_theta=spec["rope_theta"],
                      max_position_embeddings=4096, tie_word_embeddings=False,
                      initializer_range=0.2, attn_implementation="sdpa")
    torch.manual_seed(spec["model_seed"])
    return Qwen3ForCausalLM(cfg).eval()


class StubDrafter(torch.nn.Module):
    """Stands in for DFlashDraftModel in ddtree_generate: the same call signature, hidden
    states [1, block, hidden] from the noise embedding of the block and the last context
    feature through a fixed random map.  Deterministic; ignores its KV cache."""

    def __init__(self, hidden: int, seed: int = 5):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        # small weights: nearly flat draft logits, so the best-first tree takes every depth-1
        # token before going deeper and rounds accept two or more tokens
        self.proj = torch.nn.Parameter(torch.randn((hidden, hidden), generator=g) *
                                       (0.002 * hidden ** -0.5), requires_grad=False)
        self.target_layer_ids = [0]
        self.hidden = hidden

    @property
    def device(self):
        return self.proj.device

    def forward(self, target_hidden, noise_embedding, position_ids=None, past_key_values=None,
                use_cache=True, is_causal=False):
        ctx = target_hidden[:, -1:, :self.hidden].to(noise_embedding.dtype)
        return (noise_embedding + ctx) @ self.proj.to(noise_embedding.dtype)


def loop_inputs(spec: dict) -> torch.Tensor:
    rng = np.random.default_rng(spec["input_seed"])
    return torch.from_numpy(rng.integers(0, spec["vocab"] - 1, (1, spec["prompt"])).astype(np.int64))
