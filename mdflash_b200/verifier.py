"""Device-resident DDTree verify step (the hot path of ddtree_generate, ddtree.py:439-491,
without the host round trips of the reference).

    tree build   ddt_topk_tree   draft logits -> tree, ancestor bitmasks, verify ids / pos
    verify       target forward with attn_implementation="ddtree_tree" (tcgen05 kernel),
                 new K/V written in place into a TreeKVCache (no torch.cat)
    posterior    ddt_argmax      [N, V] logits -> [N] tokens
    commit       ddt_accept_compact   greedy walk + K/V compaction of every layer

Nothing in ``step`` synchronises the host; the caller reads the (small) result when it
needs it, then calls ``commit`` to set the cache length to past + accepted.

``capture`` records one step for a fixed (prefix length, budget) into a CUDA graph; a
replay re-runs every kernel of the step (tree build from the current contents of the
draft-logit buffer, the 36-layer forward, argmax, walk, compaction) with one launch
from the host, which removes the Python / launch overhead of the forward.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import attention as A
from . import kernels as K
from .cache import TreeKVCache


@dataclass
class StepResult:
    n_nodes: int
    accepted: torch.Tensor      # i64 [n_nodes] (first n_accepted valid), device
    n_accepted: torch.Tensor    # i32 [1], device
    next_token: torch.Tensor    # i64 [1], device
    posterior: torch.Tensor     # i64 [n_nodes], device
    status: torch.Tensor        # i32 [1], device: non-zero if an attention wait timed out
    logits: torch.Tensor | None = None


class TreeVerifier:
    def __init__(self, target: torch.nn.Module, cache: TreeKVCache, budget: int, depths: int,
                 vocab: int, device: torch.device | str = "cuda", keep_logits: bool = False,
                 fused: bool = False, runner=None, fused_head: bool = False,
                 posterior: torch.Tensor | None = None, walk: bool = True):
        """fused=False runs the transformers model with attn_implementation="ddtree_tree";
        fused=True runs its weights through Qwen3VerifyRunner (fused elementwise stages); a
        runner can be shared between verifiers of the same model (runner=...).  With a
        runner, fused_head=True takes the greedy posterior from the fused lm_head -> argmax
        kernel instead of cuBLAS logits + ddt_argmax (no logits then, even with
        keep_logits).  posterior: an i64 buffer (>= budget + 1) to write the greedy posterior
        into, e.g. one row of a batch; walk=False stops the step after the posterior (the
        caller walks and compacts, for instance all requests at once with
        K.accept_compact_batched)."""
        self.target = target
        self.runner = runner
        if fused and runner is None:
            from .runner import Qwen3VerifyRunner
            self.runner = Qwen3VerifyRunner(target)
        self.cache = cache
        self.budget = budget
        self.depths = depths
        self.vocab = vocab
        self.device = torch.device(device)
        self.keep_logits = keep_logits
        self.fused_head = bool(fused_head)
        self.tree = K.DeviceTree.allocate(self.device, budget, depths, vocab)
        n_cap = budget + 1
        if posterior is not None and (posterior.numel() < n_cap or posterior.dtype != torch.int64):
            raise ValueError("posterior buffer must be i64 with budget + 1 entries")
        self.posterior = (posterior.view(-1) if posterior is not None else
                          torch.zeros(n_cap, dtype=torch.int64, device=self.device))
        self.walk = bool(walk)
        self.accepted = torch.zeros(n_cap, dtype=torch.int64, device=self.device)
        self.n_accepted = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.next_token = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    @torch.inference_mode()
    def step(self, draft_logits: torch.Tensor, root_token: torch.Tensor, start: int) -> StepResult:
        """One verify step over the prefix of length ``start`` (the cache must hold
        exactly ``start`` rows).  ``draft_logits`` [depths, vocab] and ``root_token`` [1]
        are device tensors."""
        if self.cache.get_seq_length() != start:
            raise RuntimeError(f"cache holds {self.cache.get_seq_length()} rows, expected {start}")
        tree = K.topk_tree(draft_logits, self.budget, root_token, start, out=self.tree)
        return self.verify_tree(tree, start)

    @torch.inference_mode()
    def verify_tree(self, tree: K.DeviceTree, start: int) -> StepResult:
        """The step after the tree build, for a tree built elsewhere (for instance one
        request's tree of a batched build, K.topk_tree_batched) over the same prefix."""
        if self.cache.get_seq_length() != start:
            raise RuntimeError(f"cache holds {self.cache.get_seq_length()} rows, expected {start}")
        n = tree.n_nodes
        ids = tree.verify_ids[:n].view(1, n)
        pos = tree.verify_pos[:n].view(1, n)
        logits = None
        if self.runner is not None and self.fused_head:
            post = self.runner.forward_posterior(tree.verify_ids[:n], tree.verify_pos[:n],
                                                 self.cache, start, tree.anc_bits,
                                                 out=self.posterior[:n], status=self.status)
        else:
            if self.runner is not None:
                logits = self.runner.forward(tree.verify_ids[:n], tree.verify_pos[:n],
                                             self.cache, start, tree.anc_bits,
                                             status=self.status)
            else:
                with A.tree_verify(tree, start, n, status=self.status):
                    out = self.target(ids, position_ids=pos, past_key_values=self.cache,
                                      use_cache=True)
                logits = out.logits[0]
            post = K.argmax(logits, out=self.posterior[:n])
        if self.walk:
            K.accept_compact(post, tree, self.cache.kv_table(), start, accepted=self.accepted,
                             n_accepted=self.n_accepted, next_token=self.next_token, n_nodes=n)
        return StepResult(n, self.accepted, self.n_accepted, self.next_token, post, self.status,
                          logits if self.keep_logits and logits is not None else None)

    def check(self) -> None:
        """Raises DDTreeError (DDT_ERR_TIMEOUT) if an attention launch of the steps since the
        last check gave up a bounded wait (its output, and so the step's result, is then
        incomplete).  Reads the status word, so it syncs with the device."""
        K.check_status(self.status, "tree attention of the verify step")

    def commit(self, start: int, n_accepted: int) -> None:
        """Sets the cache length to start + n_accepted after the caller read the count, and
        raises if the step's attention reported a timeout (the caller has synced already)."""
        self.check()
        self.cache.crop(start + n_accepted)


class CapturedStep:
    """A verify step recorded in a CUDA graph for one prefix length.

    Inputs are read from ``draft_logits`` / ``root_token`` (device buffers owned by this
    object: copy new values in before ``replay``); outputs land in ``result``."""

    def __init__(self, verifier: TreeVerifier, start: int, warmup: int = 2,
                 time_attention: bool = False, pool=None, tree: K.DeviceTree | None = None,
                 lane: int = 0, capture_stream: torch.cuda.Stream | None = None):
        """tree=None records the whole step (tree build from ``draft_logits``); a given tree
        (built by the caller before each replay, e.g. by one batched build for many
        requests) records the step from that tree on.  Steps that may replay concurrently
        (on different streams) need different ``lane`` numbers, graph pools and capture
        streams: the lane selects this package's scratch buffers, the capture stream the
        library GEMMs' (cuBLAS keeps one workspace per stream)."""
        self.verifier = verifier
        self.start = start
        v = verifier
        self.draft_logits = torch.zeros((v.depths, v.vocab), dtype=torch.bfloat16, device=v.device)
        self.root_token = torch.zeros(1, dtype=torch.int64, device=v.device)

        def run():
            if tree is None:
                return v.step(self.draft_logits, self.root_token, start)
            return v.verify_tree(tree, start)

        side = torch.cuda.Stream(v.device)
        side.wait_stream(torch.cuda.current_stream(v.device))
        with K.WORKSPACES.lane(lane):
            with torch.cuda.stream(side):
                for _ in range(warmup):
                    run()
                    v.cache.crop(start)
            torch.cuda.current_stream(v.device).wait_stream(side)
            torch.cuda.synchronize(v.device)
            self.graph = torch.cuda.CUDAGraph()
            K.STATS.reset(time_attention=time_attention)
            with torch.cuda.graph(self.graph, pool=pool, stream=capture_stream):
                self.result = run()
        self.launches_per_replay = K.STATS.launches
        self.attn_events = list(K.STATS.attn_events)
        K.STATS.reset()
        v.cache.crop(start)

    def replay(self) -> StepResult:
        self.graph.replay()
        return self.result

    def attention_ms(self) -> list[float]:
        """Device time of each tree-attention call of the most recent replay."""
        return [a.elapsed_time(b) for a, b in self.attn_events]
