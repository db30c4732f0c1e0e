"""Device-resident DDTree verify step (the hot path of ddtree_generate, ddtree.py:439-491,
without the host round trips of the reference).

    tree build   ddt_topk_tree   draft logits -> tree, ancestor bitmasks, verify ids / pos
    verify       target forward with attn_implementation="ddtree_tree" (tcgen05 kernel),
                 new K/V written in place into a TreeKVCache (no torch.cat)
    posterior    ddt_argmax      [N, V] logits -> [N] tokens
    commit       ddt_accept_compact   greedy walk + K/V compaction of every layer

Nothing in ``step`` synchronises the host; the caller reads the (small) result when it
needs it, then calls ``commit`` to set the cache length to past + accepted.

``CapturedStep`` records one step into a CUDA graph; a replay re-runs every kernel of the
step (tree build from the current contents of the draft-logit buffer, the 36-layer forward,
argmax, walk, compaction) with one launch from the host, which removes the Python / launch
overhead of the forward.  Recorded for one prefix length, or (``max_start``) with the prefix
length in device memory, so that one graph serves every round of a decode loop whose prefix
grows (``step_device_past``).
"""
from __future__ import annotations

import dataclasses
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
    # the drafter's context features of the accepted rows (first n_accepted rows valid),
    # [budget + 1, len(feature_layers) * hidden] bf16, when the verifier was given layers
    target_hidden: torch.Tensor | None = None


class TreeVerifier:
    def __init__(self, target: torch.nn.Module, cache: TreeKVCache, budget: int, depths: int,
                 vocab: int, device: torch.device | str = "cuda", keep_logits: bool = False,
                 fused: bool = False, runner=None, fused_head: bool = False,
                 posterior: torch.Tensor | None = None, walk: bool = True,
                 feature_layers: list[int] | None = None):
        """fused=False runs the transformers model with attn_implementation="ddtree_tree";
        fused=True runs its weights through Qwen3VerifyRunner (fused elementwise stages); a
        runner can be shared between verifiers of the same model (runner=...).  With a
        runner, fused_head=True takes the greedy posterior from the fused lm_head -> argmax
        kernel instead of cuBLAS logits + ddt_argmax (no logits then, even with
        keep_logits).  posterior: an i64 buffer (>= budget + 1) to write the greedy posterior
        into, e.g. one row of a batch; walk=False stops the step after the posterior (the
        caller walks and compacts, for instance all requests at once with
        K.accept_compact_batched).  feature_layers (fused runner, with the walk): the step also
        returns the drafter's context features of the accepted rows, target_hidden =
        extract_context_feature(hidden_states, feature_layers).index_select(1, accepted)
        (ddtree.py:487), gathered on the device (ddt_gather_rows)."""
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
        self._dtrees: K.TreeBatch | None = None  # one-request batch of step_device_past
        self._kvb: K.KvBatch | None = None
        # the tree step_device_past builds into (its buffers are rewritten by every step)
        self.tree_device_past: K.DeviceTree | None = None
        self.feature_layers = list(feature_layers) if feature_layers else None
        self.features = self.target_hidden = None
        if self.feature_layers:
            if self.runner is None or not self.walk:
                raise ValueError("feature_layers needs the fused runner and the walk")
            width = len(self.feature_layers) * self.runner.hidden
            self.features = torch.zeros((n_cap, width), dtype=torch.bfloat16, device=self.device)
            self.target_hidden = torch.zeros_like(self.features)

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
                                                 out=self.posterior[:n], status=self.status,
                                                 **self._feature_args(n))
        else:
            if self.runner is not None:
                logits = self.runner.forward(tree.verify_ids[:n], tree.verify_pos[:n],
                                             self.cache, start, tree.anc_bits,
                                             status=self.status, **self._feature_args(n))
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
                          logits if self.keep_logits and logits is not None else None,
                          self._gather_features(n))

    def _feature_args(self, n: int) -> dict:
        if not self.feature_layers:
            return {}
        return {"features": self.features[:n], "feature_layers": self.feature_layers}

    def _gather_features(self, n: int):
        """The accepted rows' context features (after the walk), or None."""
        if not self.feature_layers:
            return None
        K.gather_rows(self.features[:n], self.accepted, count=self.n_accepted,
                      out=self.target_hidden)
        return self.target_hidden

    @torch.inference_mode()
    def step_device_past(self, draft_logits: torch.Tensor, root_token: torch.Tensor,
                         past_dev: torch.Tensor, max_past: int) -> StepResult:
        """One verify step whose prefix length is read from device memory (past_dev, i64 [1],
        at most max_past) by every kernel that depends on it: the tree build's verify
        positions (ddt_topk_tree_batched with one request), the K/V rows the forward writes
        (ddt_qk_norm_rope_cache_table_device_past), the attention mask
        (ddt_tree_attn_device_past, planned for max_past) and the compaction
        (ddt_accept_compact_batched).  Nothing in it depends on the host value, so a graph
        recorded from it serves every prefix length up to max_past.  Needs the fused runner
        and a cache of at least max_past + budget + 1 rows; the cache's host-side length is
        left as it is (``commit`` sets it)."""
        if self.runner is None:
            raise RuntimeError("a device-side prefix length needs the fused runner (fused=True)")
        n_cap = self.budget + 1
        if max_past < 0 or max_past + n_cap > self.cache.capacity:
            raise ValueError(f"cache holds {self.cache.capacity} rows, max_past {max_past} + "
                             f"tree window {n_cap} does not fit")
        if past_dev.dtype != torch.int64 or past_dev.numel() != 1 or not past_dev.is_cuda:
            raise ValueError("past_dev must be a device i64 [1]")
        if self._dtrees is None:
            self._dtrees = K.TreeBatch.allocate(self.device, [self.budget], self.depths,
                                                self.vocab)
            self._kvb = K.KvBatch([self.cache.kv_table()])
        root = root_token.reshape(-1)[:1]
        if root.dtype != torch.int64:
            raise ValueError("root_token must be i64")
        trees = dataclasses.replace(self._dtrees, starts=past_dev.reshape(1), root_tokens=root)
        K.topk_tree_batched(draft_logits.reshape(1, self.depths, self.vocab), trees)
        tree = trees.tree(0)
        n = tree.n_nodes
        logits = None
        if self.fused_head:
            post = self.runner.forward_posterior(tree.verify_ids[:n], tree.verify_pos[:n],
                                                 self.cache, max_past, tree.anc_bits,
                                                 out=self.posterior[:n], status=self.status,
                                                 past_dev=past_dev, **self._feature_args(n))
        else:
            logits = self.runner.forward(tree.verify_ids[:n], tree.verify_pos[:n], self.cache,
                                         max_past, tree.anc_bits, status=self.status,
                                         past_dev=past_dev, **self._feature_args(n))
            post = K.argmax(logits, out=self.posterior[:n])
        if self.walk:
            K.accept_compact_batched(self.posterior[:n_cap].view(1, n_cap), trees, self._kvb,
                                     past_dev.reshape(1), accepted=self.accepted.view(1, n_cap),
                                     n_accepted=self.n_accepted, next_token=self.next_token,
                                     status=self.status)
        self.tree_device_past = tree
        return StepResult(n, self.accepted, self.n_accepted, self.next_token, post, self.status,
                          logits if self.keep_logits and logits is not None else None,
                          self._gather_features(n) if self.walk else None)

    def check(self) -> None:
        """Raises DDTreeError (DDT_ERR_TIMEOUT) if an attention launch of the steps since the
        last check gave up a bounded wait (its output, and so the step's result, is then
        incomplete).  Reads the status word, so it syncs with the device."""
        K.check_status(self.status, "tree attention of the verify step")

    def commit(self, start: int, n_accepted: int) -> None:
        """Sets the cache length to start + n_accepted after the caller read the count, and
        raises if the step's attention reported a timeout (the caller has synced already)."""
        self.check()
        self.cache.set_seq_length(start + n_accepted)


class CapturedStep:
    """A verify step recorded in a CUDA graph, for one prefix length or (``max_start``) for
    every prefix length up to a maximum.

    Inputs are read from ``draft_logits`` / ``root_token`` (device buffers owned by this
    object: copy new values in before ``replay``); outputs land in ``result``."""

    def __init__(self, verifier: TreeVerifier, start: int, warmup: int = 2,
                 time_attention: bool = False, pool=None, tree: K.DeviceTree | None = None,
                 lane: int = 0, capture_stream: torch.cuda.Stream | None = None,
                 max_start: int | None = None, advance: bool = False):
        """tree=None records the whole step (tree build from ``draft_logits``); a given tree
        (built by the caller before each replay, e.g. by one batched build for many
        requests) records the step from that tree on.  Steps that may replay concurrently
        (on different streams) need different ``lane`` numbers, graph pools and capture
        streams: the lane selects this package's scratch buffers, the capture stream the
        library GEMMs' (cuBLAS keeps one workspace per stream).

        max_start: record TreeVerifier.step_device_past instead, with the prefix length in
        ``start_dev``; ``replay(start)`` then runs the step at any start in [0, max_start]
        (fused runner only; the attention costs what it costs at max_start, so a decode loop
        records a new step when its prefix outgrows the bucket).

        advance (with max_start): the graph also ends with ddt_advance_round, which writes the
        round's accepted tokens and next token into ``output_ids`` at the device start, logs
        the acceptance length, advances the start and makes the next token the next root:
        ``begin`` / ``run_rounds`` / ``finish`` then run several rounds with one host sync."""
        self.verifier = verifier
        self.start = start
        self.max_start = max_start
        v = verifier
        self.draft_logits = torch.zeros((v.depths, v.vocab), dtype=torch.bfloat16, device=v.device)
        self.root_token = torch.zeros(1, dtype=torch.int64, device=v.device)
        self.start_dev = None
        if max_start is not None:
            if tree is not None:
                raise ValueError("a device-side prefix length records the whole step (tree=None)")
            if not 0 <= start <= max_start:
                raise ValueError(f"start {start} outside [0, {max_start}]")
            self.start_dev = torch.full((1,), start, dtype=torch.int64, device=v.device)
        if advance and max_start is None:
            raise ValueError("advance needs max_start")
        self.advance = advance
        if advance:
            # start + accepted + 1 <= max_start + depths + 2 positions; >= 1 token per round
            self.output_ids = torch.zeros((1, max_start + v.depths + 2), dtype=torch.int64,
                                          device=v.device)
            self.acceptance = torch.zeros((1, max_start + 1), dtype=torch.int32, device=v.device)
            self.rounds_dev = torch.zeros(1, dtype=torch.int32, device=v.device)
            self._begin_start = start
            self._enqueued = 0

        def run():
            if max_start is not None:
                res = v.step_device_past(self.draft_logits, self.root_token, self.start_dev,
                                         max_start)
                if advance:
                    K.advance_round(self.start_dev, self.rounds_dev, res.n_accepted,
                                    res.accepted, v.tree_device_past.verify_ids,
                                    res.next_token, self.root_token, self.output_ids,
                                    self.acceptance, status=res.status)
                return res
            if tree is None:
                return v.step(self.draft_logits, self.root_token, start)
            return v.verify_tree(tree, start)

        side = torch.cuda.Stream(v.device)
        side.wait_stream(torch.cuda.current_stream(v.device))
        with K.WORKSPACES.lane(lane):
            with torch.cuda.stream(side):
                for _ in range(warmup):
                    if self.start_dev is not None:  # an advancing step moved it
                        self.start_dev.fill_(start)
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
        if self.start_dev is not None:
            self.start_dev.fill_(start)

    def replay(self, start: int | None = None) -> StepResult:
        """Runs the recorded step.  With max_start, ``start`` (default: the recording's) is
        the prefix length of this round: the cache must hold exactly that many rows, and
        ``commit(start, n_accepted)`` afterwards sets its new length."""
        if start is not None and start != self.start:
            if self.max_start is None:
                raise ValueError(f"step recorded for start {self.start}, not {start}")
            if not 0 <= start <= self.max_start:
                raise ValueError(f"start {start} outside [0, {self.max_start}]")
        if self.start_dev is not None:
            s = self.start if start is None else start
            if self.verifier.cache.get_seq_length() != s:
                raise RuntimeError(f"cache holds {self.verifier.cache.get_seq_length()} rows, "
                                   f"expected {s}")
            self.start_dev.fill_(s)
        self.graph.replay()
        return self.result

    def begin(self, start: int, root_token: torch.Tensor | int) -> None:
        """advance mode: the loop's first round starts at ``start`` (the cache holds exactly
        that many rows) with ``root_token``; clears the round counter."""
        if not self.advance:
            raise RuntimeError("begin / run_rounds / finish need a step recorded with advance")
        if not 0 <= start <= self.max_start:
            raise ValueError(f"start {start} outside [0, {self.max_start}]")
        if self.verifier.cache.get_seq_length() != start:
            raise RuntimeError(f"cache holds {self.verifier.cache.get_seq_length()} rows, "
                               f"expected {start}")
        self.start_dev.fill_(start)
        self.rounds_dev.zero_()
        if isinstance(root_token, torch.Tensor):
            self.root_token.copy_(root_token.reshape(-1)[:1])
        else:
            self.root_token.fill_(int(root_token))
        self._begin_start = start
        self._enqueued = 0

    def run_rounds(self, n: int) -> None:
        """advance mode: enqueues n rounds back to back (no host sync); every round reads the
        start and root the previous one left on the device.  Refuses (on the host) a count
        that could carry the start past max_start, at depths + 1 tokens per round."""
        if not self.advance:
            raise RuntimeError("begin / run_rounds / finish need a step recorded with advance")
        worst = self._begin_start + (self._enqueued + n) * (self.verifier.depths + 1)
        if worst > self.max_start:
            raise ValueError(f"{self._enqueued + n} rounds from start {self._begin_start} may "
                             f"pass max_start {self.max_start}")
        for _ in range(n):
            self.graph.replay()
        self._enqueued += n

    def finish(self) -> tuple[int, list[int]]:
        """advance mode: one sync; returns the start after the rounds run since ``begin`` and
        their acceptance lengths, sets the cache's length and raises if a kernel reported an
        error.  The committed tokens are ``output_ids[0, begin start : start + 1]`` (the last
        one is the next round's root)."""
        if not self.advance:
            raise RuntimeError("begin / run_rounds / finish need a step recorded with advance")
        start = int(self.start_dev.item())
        rounds = int(self.rounds_dev.item())
        lengths = self.acceptance[0, :rounds].tolist()
        self.verifier.commit(start, 0)
        self._begin_start = start
        self._enqueued = 0
        self.rounds_dev.zero_()
        return start, lengths

    def attention_ms(self) -> list[float]:
        """Device time of each tree-attention call of the most recent replay."""
        return [a.elapsed_time(b) for a, b in self.attn_events]
