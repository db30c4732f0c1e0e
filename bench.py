#!/usr/bin/env python
"""Benchmark of the DDTree verification hot path on B200.

Default workload, at every GPU count (one process per GPU under torchrun): a batch of 64
independent requests on a random-init Qwen3-8B-shaped target (36 layers, hidden 4096,
32 q / 8 kv heads, head_dim 128, MLP 12288, vocab 151936, bf16).  Prefix lengths are
log-uniform in 1k..32k, tree budgets uniform over {64, 128, 256, 512}, drafter logits
seeded per request (15 depths of N(0,1)*3).  A "step" verifies every request once, recorded
as one CUDA graph per rank: one batched tree-build launch for all of the rank's requests,
one 36-layer verify forward over all their tree rows (the projections and lm_head shared,
in GEMMs of at most 2048 rows; each request's K/V writes and tree attention on its own
cache, unsplit, spread over 8 streams, --lanes), one argmax over all rows, then one
batched accept walk + KV compaction of all the requests; then the result records are
all-gathered.
(--verify-batch per-request: one graph per request instead, the projections run per
request.)
Requests are assigned to ranks by longest-processing-time first; there is no other
cross-GPU traffic.
Metric: verified + accepted tokens per second over all GPUs.

  value      inputs resident in HBM; K steps bracketed by a barrier + synchronize, CUDA
             events on the step stream, max over ranks
  e2e        the same through the public API with host buffers: every request's drafter
             logits and root token are copied from pinned host memory each step, and the
             gathered result records are read back
  roofline   tree attention (the dominant kernel) at the single-request Qwen3-8B verify
             shape (prefix 8192, 257 tree rows): algorithmic FLOPs per launch over the
             launch time measured with CUDA events inside the step's graph, against the
             measured bf16 burst peak
  verify_step   sub-record: that single-request step alone (rank 0), and its decode_loop:
             16 rounds of a decode loop that replay ONE graph recorded with the prefix
             length in device memory (start advances by the accepted count every round)
  kernels    sub-record (N = 1): op-level tree build (single and batched over the mix),
             argmax, compaction (single and batched over the mix), attention and the fused
             lm_head at the same shape, L2 flushed between launches
  cpu_baseline  (N = 1) the CPU path of the reference restated (oracle): C tree build,
             torch CPU Qwen3 forward with SDPA + additive mask (fp32, all 36 layers; the
             layers share one set of weights to bound host memory, which leaves the
             compute unchanged), argmax, walk, compaction, over a bounded sample of the
             request mix

--impl reference: that CPU path alone on this host's cores (rank 0 only), one request of
the mix per step, as many steps as fit a time budget (reported).
--workload verify / attn / tree / treebatch / argmax / compact / compactbatch / lmhead /
splitkv: one sub-workload alone.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import subprocess
import sys
import tempfile
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

V = 151936
DEPTHS = 15
QWEN3_8B = dict(layers=36, hidden=4096, heads=32, kv_heads=8, head_dim=128, mlp=12288,
                vocab=V, rope_theta=1e6)
PARAMS_8B = 8.19e9
METRIC = "verified+accepted tokens/s"
VERIFY_PREFIX, VERIFY_BUDGET = 8192, 256
LOOP_ROUNDS = 16  # decode-loop rounds replayed on one graph (verify_step's decode_loop)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["requests", "verify", "attn", "tree", "treebatch",
                                           "argmax", "compact", "compactbatch", "lmhead",
                                           "splitkv"],
                    default="requests",
                    help="requests: the 64-request mix sharded over the GPUs (default); verify: "
                         "one Qwen3-8B verify step (prefix 8192, budget 256); attn / tree / "
                         "argmax / compact / lmhead: one op alone; treebatch: the batched tree "
                         "build of the request mix's trees; splitkv: attention over a prefix "
                         "sharded along the sequence")
    ap.add_argument("--prefix", type=int, default=None,
                    help="prefix length of the single-request workloads (default 8192; 131072 "
                         "for splitkv)")
    ap.add_argument("--budget", type=int, default=None,
                    help="tree budget of the single-request workloads (default 256; 512 for "
                         "splitkv)")
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--cpu-seconds", type=float, default=120.0,
                    help="time budget of the reference arm's measured steps")
    ap.add_argument("--cpu-baseline-seconds", type=float, default=20.0,
                    help="time budget of the cpu_baseline sample inside our arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="skip the verify_step / kernels sub-records")
    ap.add_argument("--tree-build", choices=["batched", "per-request"], default="batched",
                    help="requests workload: one batched tree-build launch for all of a rank's "
                         "requests per step (default), or one tree build inside each request's "
                         "graph")
    ap.add_argument("--compaction", choices=["batched", "per-request"], default="batched",
                    help="requests workload: one batched walk + compaction of all of the rank's "
                         "requests after their verify replays (default), or each request's walk "
                         "and compaction inside its graph")
    ap.add_argument("--lanes", type=int, default=0,
                    help="requests workload: streams that run requests at once: the batched "
                         "forward's per-request attention (default 8), or the per-request "
                         "graphs' replays (default 4; requests split over the lanes by "
                         "predicted cost, each lane with its own graph pool and scratch buffers)")
    ap.add_argument("--verify-batch", choices=["batched", "per-request"], default="batched",
                    help="requests workload: one verify forward over all of a rank's requests "
                         "(shared projections in fixed-size GEMM chunks, per-request K/V writes "
                         "and attention on --lanes streams), recorded as one CUDA graph; or one "
                         "graph per request")
    ap.add_argument("--gemm-chunk", type=int, default=0,
                    help="--verify-batch batched: rows per projection GEMM, every GEMM exactly "
                         "that many (the rows padded up), so that a row's result does not "
                         "depend on the other requests; 0 (default): the fewest chunks of at "
                         "most 2048 rows, each a multiple of 128, for the rank's rows")
    ap.add_argument("--batch-attn-splits", type=int, default=1,
                    help="--verify-batch batched: key splits of each request's attention "
                         "launch (1, default: one CTA per work unit and no merge, the lanes "
                         "filling the GPU with other requests' launches; 0: the library's plan)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="splitkv workload: partials travel over NVLink peer memory "
                         "(PeerExchange, default) or in an NCCL all-gather")
    ap.add_argument("--fused", type=int, default=1,
                    help="1: verify forward through the fused Qwen3 runner (default); 0: through "
                         "transformers' Qwen3 with the ddtree_tree attention plug-in")
    args = ap.parse_args()
    long_ctx = args.workload == "splitkv"
    if args.prefix is None:
        args.prefix = 131072 if long_ctx else VERIFY_PREFIX
    if args.budget is None:
        args.budget = 512 if long_ctx else VERIFY_BUDGET
    return args


def qwen3_config(attn: str, layers: int | None = None):
    from transformers import Qwen3Config
    s = QWEN3_8B
    return Qwen3Config(vocab_size=s["vocab"], hidden_size=s["hidden"], intermediate_size=s["mlp"],
                       num_hidden_layers=layers or s["layers"], num_attention_heads=s["heads"],
                       num_key_value_heads=s["kv_heads"], head_dim=s["head_dim"],
                       rope_theta=s["rope_theta"], max_position_embeddings=40960, rms_norm_eps=1e-6,
                       tie_word_embeddings=False, attn_implementation=attn)


def request_logits(seed: int) -> torch.Tensor:
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.standard_normal((DEPTHS, V)).astype(np.float32) *
                            np.float32(3.0))


def single_request_inputs(prefix: int):
    rng = np.random.default_rng(1000)
    ids = torch.from_numpy(rng.integers(0, V, (1, prefix)).astype(np.int64))
    logits = torch.from_numpy(rng.standard_normal((DEPTHS, V)).astype(np.float32) *
                              np.float32(3.0))
    return ids, logits


def tree_flops(depths: torch.Tensor, past: int, heads: int, head_dim: int) -> float:
    """4 * Hq * D * sum_i (P + |anc(i)|): QK^T and PV over each node's visible keys
    (|anc(i)| counts the node itself; the root sees P + 1 keys)."""
    anc = 1 + int(depths.sum().item()) + depths.numel()  # root: 1, node at depth d: d + 1
    n = depths.numel() + 1
    return 4.0 * heads * head_dim * (n * past + anc)


def step_roofline_ms(prefix: int, n_rows: int, peaks) -> float:
    """Lower bound of one verify step on one GPU: the slower of streaming the weights and the
    prefix K / V once (HBM) and the step's FLOPs (projections, MLP, lm_head: 2 * params * N;
    attention: 4 * Hq * D * N * P per layer) at the bf16 peak."""
    s = QWEN3_8B
    bytes_ = 2 * PARAMS_8B + 2 * s["layers"] * s["kv_heads"] * prefix * s["head_dim"] * 2
    flops = 2 * PARAMS_8B * n_rows + 4.0 * s["heads"] * s["head_dim"] * n_rows * prefix * s["layers"]
    return max(bytes_ / (peaks["hbm_gbs"] * 1e9), flops / (peaks["bf16_tflops"] * 1e12)) * 1e3


def batched_roofline_ms(requests, peaks) -> float:
    """Lower bound of one batched verify step of (prefix, rows) requests on one GPU: the
    slower of streaming the weights once and every request's prefix K / V once (HBM) and
    all the FLOPs (2 * params per row, attention 4 * Hq * D * rows * P per layer) at the bf16
    peak.  (Fixed-size GEMM chunks re-read the weights per chunk, which the bound leaves out.)"""
    s = QWEN3_8B
    kv = sum(2 * s["layers"] * s["kv_heads"] * p * s["head_dim"] * 2 for p, _ in requests)
    flops = sum(2 * PARAMS_8B * n + 4.0 * s["heads"] * s["head_dim"] * n * p * s["layers"]
                for p, n in requests)
    return max((2 * PARAMS_8B + kv) / (peaks["hbm_gbs"] * 1e9),
               flops / (peaks["bf16_tflops"] * 1e12)) * 1e3


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic(name: str):
    """DRAM bytes per launch of a kernel from the committed ncu summaries, if any."""
    path = os.path.join(ROOT, "profiles", f"{name}_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return None


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu_index)], stdout=self.tmp,
                stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.tmp.flush()
        rows = []
        with open(self.tmp.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def _gpu_index(local: int) -> int:
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    return int(visible.split(",")[local]) if visible else local


# ------------------------------------------------------------------ CPU oracle path
def cpu_target_model():
    """Qwen3-8B-shaped target for the CPU path, fp32: 36 decoder layers that share ONE set of
    random weights, and an lm_head that shares the embedding's array (the compute of every
    layer and of the lm_head is unchanged; host memory stays ~4 GB instead of 33 GB).  Each
    layer keeps its own layer index, so the KV cache has 36 layers."""
    from transformers import Qwen3ForCausalLM
    from transformers.models.qwen3.modeling_qwen3 import (Qwen3DecoderLayer, Qwen3RMSNorm,
                                                          Qwen3RotaryEmbedding)
    cfg = qwen3_config("sdpa")
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg)
        layer0 = Qwen3DecoderLayer(cfg, 0)
    layer0.to_empty(device="cpu")
    g = torch.Generator().manual_seed(0)

    def fill(t: torch.Tensor, std: float):
        # a seeded 64 Ki block tiled over the tensor (random values, cheap to make)
        blk = torch.randn(1 << 16, generator=g) * std
        flat = t.view(-1)
        full = flat.numel() // blk.numel()
        if full:
            flat[:full * blk.numel()].view(full, -1).copy_(blk.expand(full, -1))
        rest = flat.numel() - full * blk.numel()
        if rest:
            flat[full * blk.numel():].copy_(blk[:rest])

    with torch.no_grad():
        for name, p in layer0.named_parameters():
            if "norm" in name:
                p.fill_(1.0)
            else:
                fill(p, 0.02)
        sd = layer0.state_dict()
        for layer in model.model.layers:
            layer.load_state_dict(sd, assign=True)
        emb = torch.nn.Embedding(V, QWEN3_8B["hidden"])
        fill(emb.weight, 0.02)
        head = torch.nn.Linear(QWEN3_8B["hidden"], V, bias=False, device="meta")
        head.weight = emb.weight  # one [V, hidden] array for both (the lm_head GEMM is unchanged)
    model.model.embed_tokens = emb
    model.lm_head = head
    model.model.norm = Qwen3RMSNorm(QWEN3_8B["hidden"], eps=1e-6)
    model.model.rotary_emb = Qwen3RotaryEmbedding(cfg)
    return model.eval()


def cpu_request_step(model, spec, kv_cache_rows: dict):
    """One request's verify step on the CPU path: C tree build (ddtree.py:84-166 restated),
    compile with the additive mask (ddtree.py:227-267), the 36-layer fp32 forward with SDPA +
    mask, argmax (model/utils.py:28-30), walk (ddtree.py:270-281) and compaction of every
    layer (ddtree.py:284-335).  Returns (seconds, tokens = verified rows + accepted)."""
    import oracle
    from transformers import DynamicCache
    P, B = spec.prefix, spec.budget
    logits = request_logits(spec.seed).to(torch.bfloat16)  # the drafter logits the GPU sees
    root = int(np.random.default_rng(spec.seed).integers(0, V))
    k = kv_cache_rows.get(P)
    if k is None:
        g = torch.Generator().manual_seed(P)
        k = torch.randn((1, QWEN3_8B["kv_heads"], P, QWEN3_8B["head_dim"]), generator=g) * 0.5
        kv_cache_rows.clear()
        kv_cache_rows[P] = k
    cache = DynamicCache()
    for li in range(QWEN3_8B["layers"]):
        cache.update(k[..., :1, :], k[..., :1, :], li)  # creates layer li
        cache.layers[li].keys = k  # every layer's prefix is the same tensor: the verify's
        cache.layers[li].values = k  # torch.cat gives each layer its own copy
    n_cap = B + 1
    t0 = time.perf_counter()
    node_ids, depths, parents, child_maps, vis, _ = oracle.build_ddtree_tree(logits, B)
    vib = torch.empty((1, n_cap), dtype=torch.long)
    vpb = torch.empty((1, n_cap), dtype=torch.long)
    amb = torch.zeros((1, 1, n_cap, P + n_cap), dtype=torch.float32)
    tvb = torch.empty((n_cap, n_cap), dtype=torch.bool)
    vi, vp, am, _, n = oracle.compile_ddtree_tree(root, P, node_ids, depths, vis, P,
                                                  torch.float32, None, vib, vpb, amb, tvb, 0, 0)
    with torch.inference_mode():
        out = model(vi, position_ids=vp, attention_mask=am, past_key_values=cache, use_cache=True)
        post = oracle.argmax(out.logits[0])
        acc, nxt = oracle.follow_verified_tree(child_maps, post)
        layers_np = [(l.keys.numpy(), l.values.numpy()) for l in cache.layers]
        oracle.compact_dynamic_cache(layers_np, P, acc)
    return time.perf_counter() - t0, n + len(acc)


def cpu_sample(n_requests: int, budget_s: float, warmup: int, max_steps: int):
    """Runs requests of the mix (seeded order) one per step on the host cores: `warmup`
    untimed steps, then measured steps until `budget_s` seconds are spent (at least one, at
    most max_steps).  Returns tokens/s over the measured steps and what was run."""
    from mdflash_b200 import sharding as S
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    t_build = time.perf_counter()
    model = cpu_target_model()
    t_build = time.perf_counter() - t_build
    specs = S.request_specs(n_requests, seed=0)
    order = np.random.default_rng(7).permutation(len(specs))
    kv_rows: dict = {}
    i = 0
    for _ in range(warmup):
        cpu_request_step(model, specs[order[i % len(order)]], kv_rows)
        i += 1
    times, tokens, ran = [], 0, []
    spent = 0.0
    while len(times) < max(1, max_steps) and (not times or spent < budget_s):
        sp = specs[order[i % len(order)]]
        dt, tok = cpu_request_step(model, sp, kv_rows)
        times.append(dt)
        tokens += tok
        ran.append((sp.index, sp.prefix, sp.budget))
        spent += dt
        i += 1
    return {"value": tokens / sum(times), "seconds": sum(times), "steps": len(times),
            "ms_per_step": 1e3 * sum(times) / len(times), "threads": threads,
            "model_build_s": t_build,
            "sample": f"{len(times)} requests of the {n_requests}-request mix after {warmup} "
                      f"warm-up, one full verify step each (36 fp32 decoder layers sharing one "
                      f"weight set, SDPA + additive mask; C tree build, argmax, walk, "
                      f"compaction of all layers); requests (index, prefix, budget): {ran}"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    r = cpu_sample(args.requests, args.cpu_seconds, min(args.warmup, 1), args.steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": r["steps"], "requested_steps": args.steps,
        "warmup": min(args.warmup, 1), "ms_per_step": r["ms_per_step"],
        "step": "one request of the mix (the CPU path verifies requests one at a time)",
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": requests_config(args, args.gpus),
        "cpu_baseline": {"value": r["value"], "unit": "tokens/s", "cores": r["threads"],
                         "kind": "port", "sample": r["sample"]},
        "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "timed_seconds": r["seconds"], "model_build_s": r["model_build_s"],
    }
    print(json.dumps(line), flush=True)


def requests_config(args, n):
    return {"workload": f"{args.requests} independent DDTree verify requests on a Qwen3-8B-shaped "
                        "target (36 layers, bf16): prefix log-uniform 1k-32k, budget in "
                        "{64,128,256,512}, 15 drafted depths; one verify step of every request",
            "model": "Qwen3-8B shape, random init", "global_batch": args.requests,
            "seq_len": "1024-32768 (log-uniform)", "parallelism": f"request-dp{n} (LPT)",
            "l2": "inputs larger than L2: 16 GB of weights streamed per GEMM row chunk, "
                  "86 GB of prefix K/V"}


# ------------------------------------------------------------------------ our arm
def _dist_setup():
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    return world, rank, local, dev


def gpu_model(dev, attn):
    from transformers import Qwen3ForCausalLM
    torch.manual_seed(0)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev), torch.inference_mode():
        model = Qwen3ForCausalLM(qwen3_config(attn)).eval()
    torch.set_default_dtype(prev)
    return model


def _fill_prefix(cache, prefix: int, g: torch.Generator):
    for layer in cache.layers:
        layer.k_buf[..., :prefix, :].normal_(0.0, 1.0, generator=g)
        layer.v_buf[..., :prefix, :].normal_(0.0, 1.0, generator=g)
        layer.length = prefix
        layer.keys = layer.k_buf[..., :prefix, :]
        layer.values = layer.v_buf[..., :prefix, :]


def _batched_verify(args, dev, runner, specs, mine, trees, dev_logits, host_logits, host_roots,
                    g, rank, lanes):
    """--verify-batch batched: every request of this rank in ONE verify step, recorded as one
    CUDA graph: the batched tree build, a gather of the tree rows into one row block (request
    after request), Qwen3VerifyRunner.forward_batch (projections over all rows in GEMMs of
    --gemm-chunk rows, K/V writes and tree attention per request on `lanes` streams), one
    argmax over all rows scattered back per request, and the batched walk + compaction.
    Returns (one_step, check_statuses, records, launches per step, execution)."""
    from mdflash_b200 import kernels as K
    from mdflash_b200 import sharding as S
    from mdflash_b200.cache import TreeKVCache
    from mdflash_b200.runner import gemm_chunk
    R = len(mine)
    records = torch.full((R, S.RECORD_LEN), -1, dtype=torch.int64, device=dev)
    if R == 0:
        return (lambda e2e: S.gather_results(records)), (lambda: None), records, 0, "no requests"
    mb1 = trees.max_budget + 1
    caches, segments, pasts, ancs, src = [], [], [], [], []
    off = 0
    for j, i in enumerate(mine):
        sp = specs[i]
        n = 1 + K.expected_node_count(DEPTHS, V, sp.budget)
        cache = TreeKVCache(QWEN3_8B["layers"], sp.prefix + sp.budget + 1 + 64).allocate(
            QWEN3_8B["kv_heads"], QWEN3_8B["head_dim"], torch.bfloat16, dev)
        _fill_prefix(cache, sp.prefix, g.manual_seed(1000 + sp.index))
        caches.append(cache)
        segments.append((off, n))
        pasts.append(sp.prefix)
        ancs.append(trees.anc_bits[j, :n])
        src += [j * mb1 + t for t in range(n)]
        off += n
    T = off
    chunk = args.gemm_chunk if args.gemm_chunk > 0 else gemm_chunk(T)
    t_pad = -(-T // chunk) * chunk
    idx = torch.tensor(src, dtype=torch.int64, device=dev)
    ids_buf = torch.zeros(t_pad, dtype=torch.int64, device=dev)
    pos_buf = torch.zeros(t_pad, dtype=torch.int64, device=dev)
    post_cat = torch.zeros(T, dtype=torch.int64, device=dev)
    posteriors = torch.zeros((R, mb1), dtype=torch.int64, device=dev)
    kvb = K.KvBatch([c.kv_table() for c in caches])
    past_dev = torch.tensor(pasts, dtype=torch.int64, device=dev)
    b_acc = torch.zeros((R, mb1), dtype=torch.int64, device=dev)
    b_n = torch.zeros(R, dtype=torch.int32, device=dev)
    b_next = torch.zeros(R, dtype=torch.int64, device=dev)
    status = K.attention_status(dev)

    def step():
        K.topk_tree_batched(dev_logits, trees)
        torch.index_select(trees.verify_ids.view(-1), 0, idx, out=ids_buf[:T])
        torch.index_select(trees.verify_pos.view(-1), 0, idx, out=pos_buf[:T])
        logits = runner.forward_batch(ids_buf, pos_buf, segments, caches, pasts, ancs,
                                      status=status, chunk=chunk, lanes=lanes,
                                      kv_splits=args.batch_attn_splits)
        K.argmax(logits[:T], out=post_cat)
        posteriors.view(-1).index_copy_(0, idx, post_cat)
        K.accept_compact_batched(posteriors, trees, kvb, past_dev, b_acc, b_n, b_next,
                                 status=status)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side), torch.inference_mode():
        for _ in range(2):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    K.STATS.reset()
    with torch.inference_mode(), torch.cuda.graph(graph):
        step()
    launches = K.STATS.launches
    K.STATS.reset()
    for j, i in enumerate(mine):
        records[j, :3] = torch.tensor([specs[i].index, rank, segments[j][1]])
        records[j, 5] = 0
    m_path = min(S.MAX_PATH, mb1)
    nn = torch.tensor([n for _, n in segments], device=dev)
    path_cols = torch.arange(m_path, device=dev)[None, :] < nn[:, None]
    # everything the recorded graph reads or writes outside its own pool stays referenced by
    # the returned closures for as long as the graph is replayed
    live = (caches, ancs, idx, ids_buf, pos_buf, post_cat, posteriors, kvb, past_dev, status)

    def one_step(e2e: bool):
        assert live is not None
        if e2e:  # this step's inputs from pinned host memory
            dev_logits.copy_(host_logits, non_blocking=True)
            trees.root_tokens.copy_(host_roots, non_blocking=True)
        graph.replay()
        records[:, 3] = b_n
        records[:, 4] = b_next
        records[:, 6:6 + m_path] = torch.where(path_cols, b_acc[:, :m_path], -1)
        return S.gather_results(records)

    def check_statuses():
        if int(status.item()) != 0:
            raise RuntimeError(f"device status {int(status.item()):#x} in the batched verify")

    execution = (f"one CUDA graph per step for the rank's {R} requests: batched tree build, one "
                 f"36-layer verify forward over their {T} tree rows (projections in GEMMs of "
                 f"{chunk} rows, {t_pad - T} padding rows; K/V writes and tree attention per "
                 f"request on {lanes} streams), argmax, batched walk + compaction; records "
                 "all-gathered per step")
    return one_step, check_statuses, records, launches, execution


def run_requests(args):
    """The default workload (see the module docstring); prints the JSON line on rank 0."""
    import torch.distributed as dist

    from mdflash_b200 import attention as A
    from mdflash_b200 import kernels as K
    from mdflash_b200 import sharding as S
    from mdflash_b200.cache import TreeKVCache
    from mdflash_b200.runner import Qwen3VerifyRunner
    from mdflash_b200.verifier import CapturedStep, TreeVerifier

    world, rank, local, dev = _dist_setup()
    K._lib.load(build_if_missing=False)
    attn = A.register()
    model = gpu_model(dev, attn)
    runner = Qwen3VerifyRunner(model)
    specs = S.request_specs(args.requests, seed=0)
    assignment = S.assign_requests([S.request_cost(s) for s in specs], world)
    mine = assignment[rank]
    lanes = args.lanes if args.lanes > 0 else (8 if args.verify_batch == "batched" else 4)
    pools = [torch.cuda.graph_pool_handle() for _ in range(lanes)]
    streams = [torch.cuda.Stream(dev) for _ in range(lanes)] if lanes > 1 else None
    cap_streams = [torch.cuda.Stream(dev) for _ in range(lanes)] if lanes > 1 else None
    caps = []
    g = torch.Generator(device=dev)
    batched = args.tree_build == "batched"
    # every request's drafter logits and root token, pinned on the host and resident on the
    # device ([R, depths, V]); the batched build reads them all in one launch
    host_logits = torch.stack([request_logits(specs[i].seed).to(torch.bfloat16)
                               for i in mine]).pin_memory() if mine else None
    host_roots = torch.tensor([int(np.random.default_rng(specs[i].seed).integers(0, V))
                               for i in mine], dtype=torch.int64).pin_memory()
    dev_logits = host_logits.to(dev) if mine else None
    trees = K.TreeBatch.allocate(dev, [specs[i].budget for i in mine], DEPTHS, V) if mine else None
    if mine:
        trees.starts.copy_(torch.tensor([specs[i].prefix for i in mine]))
        trees.root_tokens.copy_(host_roots)
        if batched:
            K.topk_tree_batched(dev_logits, trees)  # the trees the captured steps start from
    # lanes get equal shares of the predicted work (longest-processing-time first over the
    # request cost model); within a lane the longest requests go first, and the replay order
    # interleaves the lanes so that all of them start at once.  A lane's graphs share one
    # pool, so they are captured in the order they are replayed.
    lane_lists = S.assign_requests([S.request_cost(specs[i]) for i in mine], lanes)
    lane_of = {}
    for ln, lst in enumerate(lane_lists):
        lst.sort(key=lambda j: (-S.request_cost(specs[mine[j]]), j))
        for j in lst:
            lane_of[j] = ln
    order = [lst[t] for t in range(max((len(x) for x in lane_lists), default=0))
             for lst in lane_lists if t < len(lst)]
    if args.verify_batch == "batched":
        bcompact = True
        one_step, check_statuses, records, launches_per_step, execution = \
            _batched_verify(args, dev, runner, specs, mine, trees, dev_logits, host_logits,
                            host_roots, g, rank, lanes)
        caps = []
    else:
        # the batched walk reads the batched build's trees
        bcompact = args.compaction == "batched" and batched
        posteriors = (torch.zeros((len(mine), trees.max_budget + 1), dtype=torch.int64, device=dev)
                      if mine else None)
        caps = [None] * len(mine)
        for j in order:
            sp = specs[mine[j]]
            ln = lane_of[j]
            cache = TreeKVCache(QWEN3_8B["layers"], sp.prefix + sp.budget + 1 + 64).allocate(
                QWEN3_8B["kv_heads"], QWEN3_8B["head_dim"], torch.bfloat16, dev)
            # random prefix K / V seeded per request (the verify work does not depend on the
            # values; the results then do not depend on the rank or the capture order)
            _fill_prefix(cache, sp.prefix, g.manual_seed(1000 + sp.index))
            ver = TreeVerifier(model, cache, sp.budget, DEPTHS, V, dev, runner=runner,
                               posterior=posteriors[j] if bcompact else None, walk=not bcompact)
            cap = CapturedStep(ver, sp.prefix, warmup=1, pool=pools[ln],
                               tree=trees.tree(j) if batched else None, lane=ln,
                               capture_stream=cap_streams[ln] if cap_streams else None)
            cap.draft_logits.copy_(dev_logits[j])
            cap.root_token.copy_(trees.root_tokens[j:j + 1])
            caps[j] = (sp, cap)
        records = torch.full((len(caps), S.RECORD_LEN), -1, dtype=torch.int64, device=dev)
        for j, (sp, cap) in enumerate(caps):
            records[j, :3] = torch.tensor([sp.index, rank, cap.result.n_nodes])
            records[j, 5] = 0
        if bcompact and caps:
            kvb = K.KvBatch([cap.verifier.cache.kv_table() for _, cap in caps])
            K.accept_compact_batched(posteriors, trees, kvb, [sp.prefix for sp, _ in caps])
            past_dev = torch.tensor([sp.prefix for sp, _ in caps], dtype=torch.int64, device=dev)
            b_acc = torch.zeros((len(caps), trees.max_budget + 1), dtype=torch.int64, device=dev)
            b_n = torch.zeros(len(caps), dtype=torch.int32, device=dev)
            b_next = torch.zeros(len(caps), dtype=torch.int64, device=dev)
            m_path = min(S.MAX_PATH, trees.max_budget + 1)
            # path columns a request's record holds: min(MAX_PATH, its node count), the rest -1
            nn = torch.tensor([cap.result.n_nodes for _, cap in caps], device=dev)
            path_cols = torch.arange(m_path, device=dev)[None, :] < nn[:, None]

        def one_step(e2e: bool):
            if e2e and batched and caps:  # this step's inputs from pinned host memory
                dev_logits.copy_(host_logits, non_blocking=True)
                trees.root_tokens.copy_(host_roots, non_blocking=True)
            if batched and caps:
                K.topk_tree_batched(dev_logits, trees)
            main = torch.cuda.current_stream(dev)
            if streams:
                for st in streams:
                    st.wait_stream(main)
            for j in order:
                sp, cap = caps[j]
                with torch.cuda.stream(streams[lane_of[j]] if streams else main):
                    if e2e and not batched:
                        cap.draft_logits.copy_(host_logits[j], non_blocking=True)
                        cap.root_token.copy_(host_roots[j:j + 1], non_blocking=True)
                    r = cap.replay()
                    if not bcompact:
                        # record on the device: [index, rank, n_nodes, n_accepted, next, 0, path...]
                        records[j, 3] = r.n_accepted[0]
                        records[j, 4] = r.next_token[0]
                        m = min(S.MAX_PATH, r.n_nodes)
                        records[j, 6:6 + m] = r.accepted[:m]
            if streams:
                for st in streams:
                    main.wait_stream(st)
            if bcompact and caps:
                # every request's walk and compaction in one batched launch after the replays
                K.accept_compact_batched(posteriors, trees, kvb, past_dev, b_acc, b_n, b_next)
                records[:, 3] = b_n
                records[:, 4] = b_next
                records[:, 6:6 + m_path] = torch.where(path_cols, b_acc[:, :m_path], -1)
            return S.gather_results(records)

        def check_statuses():
            st = torch.stack([cap.verifier.status for _, cap in caps])
            if int(st.abs().sum().item()) != 0:
                raise RuntimeError("a tree-attention launch reported a bounded-wait timeout")

        launches_per_step = (sum(cap.launches_per_replay for _, cap in caps)
                             + (1 if batched and caps else 0) + (2 if bcompact and caps else 0))
        execution = (("one batched tree-build launch for the rank's requests, then "
                      "one CUDA-graph replay per request (36-layer fused verify forward, argmax"
                      + (f") on {lanes} lanes, then one batched walk + compaction" if bcompact
                         else ", accept walk + compaction)") if batched else
                      "one CUDA-graph replay per request (tree build, 36-layer fused verify "
                      "forward, argmax, accept walk + compaction)") +
                     "; records all-gathered per step")
    for _ in range(args.warmup):
        one_step(False)
    torch.cuda.synchronize()
    check_statuses()

    def timed(e2e: bool):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        allrec = None
        host_rec = None
        for _ in range(args.steps):
            allrec = one_step(e2e)
            if e2e:
                host_rec = allrec.cpu()  # the step's results on the host (syncs)
        ev1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = torch.tensor([ev0.elapsed_time(ev1) / args.steps], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item(), (host_rec if host_rec is not None else allrec.cpu())

    with ClockSampler(_gpu_index(local)) as clocks:
        ms, allrec = timed(False)
    clock_summary = clocks.summary()
    tokens = int((allrec[:, 2] + allrec[:, 3]).sum())
    value = tokens / (ms / 1e3)
    for _ in range(args.warmup):
        one_step(True)
    e2e_ms, e2e_rec = timed(True)
    e2e_tokens = int((e2e_rec[:, 2] + e2e_rec[:, 3]).sum())
    check_statuses()
    h2d = (host_logits.numel() * host_logits.element_size() + host_roots.numel() * 8) if mine else 0
    d2h = int(allrec.numel()) * 8
    launches = launches_per_step * args.steps
    sums = torch.tensor([float(h2d), float(launches)], device=dev)
    if world > 1:
        dist.all_reduce(sums, op=dist.ReduceOp.SUM)
    peaks, peak_kind = measured_peaks()
    # lower bound of the whole job: each GPU's requests back to back at their step roofline
    if args.verify_batch == "batched":
        bound = max(batched_roofline_ms([(specs[i].prefix, specs[i].budget + 1) for i in a],
                                        peaks) for a in assignment)
        bound_kind = ("max(HBM: weights once + every request's prefix K/V once, bf16 FLOPs of "
                      "all rows) for the slowest rank's batched step")
    else:
        bound = max(sum(step_roofline_ms(specs[i].prefix, specs[i].budget + 1, peaks)
                        for i in a) for a in assignment)
        bound_kind = ("max(HBM: weights + prefix K/V once, bf16 FLOPs) per request, the slowest "
                      "rank's requests back to back")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded request mix, random prefix K/V, N(0,1)*3 drafter logits, "
                "random-init Qwen3-8B-shaped weights",
        "config": requests_config(args, world),
        "e2e": {"value": e2e_tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(sums[0].item()), "d2h_bytes_per_step": d2h * world,
                "ms_per_step": e2e_ms},
        "gpu_launches": int(sums[1].item()),
        "tokens_per_step": tokens,
        # digest of the gathered result records (accepted paths, next tokens) without their
        # rank field: the same at every GPU count and --lanes / --tree-build setting (for one
        # --verify-batch / --batch-attn-splits choice: their attention plans round apart), since
        # every request's step is deterministic
        "records_digest": hashlib.sha1(
            allrec.index_fill(1, torch.tensor([1]), 0).numpy().tobytes()).hexdigest()[:16],
        "requests_per_rank": [len(a) for a in assignment],
        "step_roofline": {"bound": bound_kind, "ms": bound, "frac": bound / ms, "peak_source": peak_kind},
        "execution": execution,
        "verify_batch": args.verify_batch,
        "tree_build": args.tree_build,
        "compaction": "batched" if bcompact else "per-request",
        "lanes": lanes,
    }
    del caps
    one_step = check_statuses = None  # the batched step's graph, caches and buffers
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if rank == 0 and not args.no_subrecords:
        with ClockSampler(_gpu_index(local)) as sub_clocks:
            sub = verify_step(args, model, runner, dev, steps=max(3, min(args.steps, 20)),
                              warmup=args.warmup)
        sub["clocks"] = sub_clocks.summary()
        line["verify_step"] = sub
        line["roofline"] = dict(sub["roofline"], clocks=sub["clocks"])
        if world == 1:
            line["kernels"] = kernel_table(dev, args)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_sample(args.requests, args.cpu_baseline_seconds, 0, 1 << 30)
        line["cpu_baseline"] = {"value": r["value"], "unit": "tokens/s", "cores": r["threads"],
                                "kind": "port", "sample": r["sample"]}
    line["clocks"] = clock_summary
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def verify_step(args, model, runner, dev, steps: int, warmup: int, prefix: int = VERIFY_PREFIX,
                budget: int = VERIFY_BUDGET):
    """One Qwen3-8B verify step (causal prefill of `prefix` tokens on the same kernels, then a
    `budget`-node tree), replayed as one CUDA graph; the tree-attention launches are bracketed
    by CUDA events inside the graph."""
    from mdflash_b200 import kernels as K
    from mdflash_b200.cache import TreeKVCache
    from mdflash_b200.verifier import CapturedStep, TreeVerifier
    ids, logits = single_request_inputs(prefix)
    P, B = prefix, budget
    cache = TreeKVCache(QWEN3_8B["layers"], P + B + 1 + LOOP_ROUNDS * (DEPTHS + 1)).allocate(
        QWEN3_8B["kv_heads"], QWEN3_8B["head_dim"], torch.bfloat16, dev)
    verifier = TreeVerifier(model, cache, B, DEPTHS, V, dev, runner=runner)
    with torch.inference_mode():
        out_logits = runner.forward(ids[0].to(dev), torch.arange(P, device=dev), cache, 0, None,
                                    causal=True)
        root_dev = K.argmax(out_logits[-1:]).view(1).clone()
        del out_logits
    draft_dev = logits.to(torch.bfloat16).to(dev)
    n_nodes = 1 + K.expected_node_count(DEPTHS, V, B)
    for _ in range(warmup):
        verifier.step(draft_dev, root_dev, P)
        cache.crop(P)  # every step verifies the same prefix (the commit is undone)
    cap = CapturedStep(verifier, P, warmup=1, time_attention=True)
    cap.draft_logits.copy_(draft_dev)
    cap.root_token.copy_(root_dev)
    for _ in range(warmup):
        cap.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    ev0.record()
    for _ in range(steps):
        res = cap.replay()
    ev1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    verifier.check()
    ms = ev0.elapsed_time(ev1) / steps
    attn_ms = cap.attention_ms()
    n_acc = int(res.n_accepted.item())
    depths = verifier.tree.node_depths[:n_nodes - 1].cpu()
    peaks, peak_kind = measured_peaks()
    flops = tree_flops(depths, P, QWEN3_8B["heads"], QWEN3_8B["head_dim"])
    attn_mean = float(np.mean(attn_ms))
    achieved = flops / (attn_mean / 1e3) / 1e12
    peak = float(peaks["bf16_tflops"])
    traffic = profile_traffic("tree_attn")
    step_bound = step_roofline_ms(P, n_nodes, peaks)
    launches = cap.launches_per_replay
    del cap
    loop = decode_loop(verifier, draft_dev, root_dev, P, LOOP_ROUNDS, warmup, ms)
    return {
        "workload": f"Qwen3-8B-shaped verify step: 36 layers, prefix {P}, {B}-node best-first tree "
                    "(15 depths), bf16, one CUDA-graph replay per step",
        "value": (n_nodes + n_acc) / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
        "steps": steps, "verified_per_step": n_nodes, "accepted_per_step": n_acc,
        "launches_per_step": launches,
        "attention_share": attn_mean * QWEN3_8B["layers"] / ms,
        "step_roofline": {"ms": step_bound, "frac": step_bound / ms},
        "roofline": {"kernel": "ddt_tree_attn (+ its split merge), one launch per layer, inside "
                               "the verify step's graph",
                     "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak,
                     "peak_source": f"{peak_kind} bf16 burst (MEASURED_PEAKS.json bf16_tflops): "
                                    "the kernel runs ~50 us at a time",
                     "flops_per_launch": flops, "launch_ms": attn_mean,
                     "launches_timed": len(attn_ms),
                     "traffic": traffic.get("bytes_per_launch") if traffic else None},
        "decode_loop": loop,
    }


def decode_loop(verifier, draft_dev, root_dev, P: int, rounds: int, warmup: int,
                fixed_ms: float) -> dict:
    """`rounds` rounds of a decode loop (ddtree.py:417-506) on ONE CUDA graph recorded with
    the prefix length in device memory (CapturedStep(max_start=...)): each round replays it at
    the current start, reads the accepted count (the loop's one host sync per round),
    commits, advances start by the accepted count and feeds the next token back as the root.
    Timed with CUDA events around all rounds, host gaps included; the cache is restored to
    the prefix afterwards.  Then the same rounds enqueued back to back with one host sync
    (the recorded step advances its own start and root on the device, ddt_advance_round)."""
    from mdflash_b200.verifier import CapturedStep
    cache = verifier.cache
    max_start = P + rounds * (DEPTHS + 1)
    cap = CapturedStep(verifier, P, warmup=1, max_start=max_start, advance=True)
    cap.draft_logits.copy_(draft_dev)

    def run():
        cap.root_token.copy_(root_dev)
        start, acc = P, []
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(rounds):
            res = cap.replay(start)
            k = int(res.n_accepted.item())
            verifier.commit(start, k)
            acc.append(k)
            start += k
            cap.root_token.copy_(res.next_token)
        ev1.record()
        torch.cuda.synchronize()
        cache.set_seq_length(P)
        return ev0.elapsed_time(ev1), acc, res.n_nodes

    def run_device():
        cap.begin(P, root_dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        cap.run_rounds(rounds)
        ev1.record()
        _, lengths = cap.finish()
        cache.set_seq_length(P)
        return ev0.elapsed_time(ev1), lengths

    for _ in range(warmup):
        run()
        run_device()
    total_ms, acc, n_nodes = run()
    dev_ms, dev_acc = run_device()
    del cap
    ms = total_ms / rounds
    return {"rounds": rounds, "graphs_recorded": 1, "max_start": max_start,
            "start_first": P, "start_last": P + sum(acc) - acc[-1],
            "accepted_per_round": float(np.mean(acc)), "ms_per_round": ms,
            "value": (rounds * n_nodes + sum(acc)) / (total_ms / 1e3), "unit": "tokens/s",
            "vs_fixed_prefix_step": ms / fixed_ms,
            "device_advanced": {"ms_per_round": dev_ms / rounds, "host_syncs": 1,
                                "vs_fixed_prefix_step": dev_ms / rounds / fixed_ms,
                                "same_acceptance_as_host_loop": dev_acc == acc}}


# ------------------------------------------------------------ op-level measurements
def _timed_launches(fn, steps: int, warmup: int, dev) -> float:
    """Mean device time (ms) of `fn` over `steps` launches, each bracketed by CUDA events,
    with a 256 MB buffer written before each launch (L2 flushed)."""
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    torch.cuda.nvtx.range_push("timed")
    for _ in range(steps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        times.append((a, b))
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    return float(np.mean([a.elapsed_time(b) for a, b in times]))


def attn_inputs(prefix: int, budget: int, seed: int = 0):
    """Tree attention op inputs: Hq=32, Hkv=8, D=128, Q/K/V ~ N(0,1)/sqrt(128), parents of
    a seeded random tree (BFS growth, Geometric(0.5) child counts, depth <= 16)."""
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import inputs as gin
    n = budget + 1
    g = torch.Generator().manual_seed(seed)
    sc = 1.0 / math.sqrt(128)
    q = (torch.randn((n, 32, 128), generator=g) * sc).to(torch.bfloat16)
    k = (torch.randn((8, prefix + n, 128), generator=g) * sc).to(torch.bfloat16)
    v = (torch.randn((8, prefix + n, 128), generator=g) * sc).to(torch.bfloat16)
    parents = gin.random_tree(n, seed + 1)
    return q, k, v, parents


def anc_bits_host(parents: np.ndarray) -> np.ndarray:
    n = parents.shape[0]
    words = (n + 31) // 32
    bits = np.zeros((n, words), np.uint32)
    for i in range(n):
        j = i
        while j >= 0:
            bits[i, j // 32] |= np.uint32(1 << (j % 32))
            j = int(parents[j]) if j > 0 else -1
    return bits


def attn_flops(parents: np.ndarray, past: int) -> float:
    n = parents.shape[0]
    depth = np.zeros(n, np.int64)
    for i in range(1, n):
        depth[i] = depth[parents[i]] + 1
    return 4.0 * 32 * 128 * float(n * past + int((depth + 1).sum()))


def measure_attn(dev, prefix, budget, steps, warmup):
    from mdflash_b200 import kernels as K
    q, k, v, parents = attn_inputs(prefix, budget)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    bits = torch.from_numpy(anc_bits_host(parents).view(np.int32)).to(dev)
    out = K.tree_attention(qd, kd, vd, bits, prefix)
    ms = _timed_launches(lambda: K.tree_attention(qd, kd, vd, bits, prefix, out=out), steps,
                         warmup, dev)
    K.check_status(K.attention_status(dev))
    flops = attn_flops(parents, prefix)
    peaks, kind = measured_peaks()
    tflops = flops / (ms / 1e3) / 1e12
    return {"ms": ms, "tflops": tflops, "frac": tflops / peaks["bf16_tflops"],
            "peak": peaks["bf16_tflops"], "peak_source": f"{kind} bf16 burst",
            "flops_per_launch": flops,
            "kv_splits": K.attn_splits(budget + 1, 32, 8, prefix),
            "shape": f"Hq 32 / Hkv 8, D 128, prefix {prefix}, {budget + 1} tree rows"}


def measure_tree(dev, budget, steps, warmup):
    from mdflash_b200 import kernels as K
    _, logits = single_request_inputs(16)
    x = logits.to(torch.bfloat16).to(dev)
    root = torch.zeros(1, dtype=torch.int64, device=dev)
    tree = K.topk_tree(x, budget, root, VERIFY_PREFIX)
    ms = _timed_launches(lambda: K.topk_tree(x, budget, root, VERIFY_PREFIX, out=tree), steps,
                         warmup, dev)
    nbytes = x.numel() * x.element_size()
    peaks, kind = measured_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"ms": ms, "gbs": gbs, "frac": gbs / peaks["hbm_gbs"], "peak": peaks["hbm_gbs"],
            "peak_source": kind, "bytes_per_launch": nbytes,
            "shape": f"15 x {V} bf16 drafter logits, budget {budget}",
            "node_count": int(tree.node_count.item())}


def measure_tree_batched(dev, n_requests, steps, warmup):
    """One ddt_topk_tree_batched launch over the request mix's drafter logits (n_requests x 15
    x V bf16, the mix's budgets)."""
    from mdflash_b200 import kernels as K
    from mdflash_b200 import sharding as S
    specs = S.request_specs(n_requests, seed=0)
    x = torch.stack([request_logits(sp.seed).to(torch.bfloat16) for sp in specs]).to(dev)
    trees = K.TreeBatch.allocate(dev, [sp.budget for sp in specs], DEPTHS, V)
    trees.starts.copy_(torch.tensor([sp.prefix for sp in specs]))
    ms = _timed_launches(lambda: K.topk_tree_batched(x, trees), steps, warmup, dev)
    nbytes = x.numel() * x.element_size()
    peaks, kind = measured_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"ms": ms, "gbs": gbs, "frac": gbs / peaks["hbm_gbs"], "peak": peaks["hbm_gbs"],
            "peak_source": kind, "bytes_per_launch": nbytes, "requests": n_requests,
            "shape": f"{n_requests} requests x 15 x {V} bf16 drafter logits, budgets of the mix",
            "nodes": int(trees.node_count.sum().item())}


def measure_argmax(dev, rows, steps, warmup):
    from mdflash_b200 import kernels as K
    g = torch.Generator(device=dev).manual_seed(0)
    logits = torch.randn((rows, V), generator=g, device=dev).mul_(3).to(torch.bfloat16)
    out = torch.empty(rows, dtype=torch.int64, device=dev)
    ms = _timed_launches(lambda: K.argmax(logits, out=out), steps, warmup, dev)
    # what a plain device copy of the same bytes reaches, timed the same way: the stream
    # ceiling of a launch this size (copy bytes counted read + write, as the HBM peak is)
    dst = torch.empty_like(logits)
    ms_copy = _timed_launches(lambda: dst.copy_(logits), steps, warmup, dev)
    ref = logits.float().argmax(-1)
    if not torch.equal(out, ref):
        raise RuntimeError("argmax disagrees with torch.argmax on the bench data")
    nbytes = logits.numel() * logits.element_size()
    peaks, kind = measured_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    copy_gbs = 2 * nbytes / (ms_copy / 1e3) / 1e9
    return {"ms": ms, "gbs": gbs, "frac": gbs / peaks["hbm_gbs"], "peak": peaks["hbm_gbs"],
            "peak_source": kind, "bytes_per_launch": nbytes,
            "same_size_copy": {"ms": ms_copy, "gbs": copy_gbs,
                               "frac": copy_gbs / peaks["hbm_gbs"]},
            "shape": f"[{rows}, {V}] bf16 verify logits, N(0,1)*3"}


def measure_compact(dev, prefix, budget, steps, warmup):
    """Accept walk + KV compaction alone on the Qwen3-8B cache shape (36 layers x K, V
    [1, 8, P + N, 128] bf16) with a forced accepted path: the posterior follows the tree
    from the root to its deepest node (the drafter logits make the tree reach all 15
    depths), so a 16-row path is accepted and each layer's K and V move one row per
    accepted node not already in place.  GB/s of the algorithmic bytes (read + write of
    every moved row) over the launch time."""
    from mdflash_b200 import kernels as K
    layers, hkv, d = 36, 8, 128
    _, logits = single_request_inputs(16)
    # one token per depth lifted to about the log-sum-exp of the rest (log-prob ~ -0.7), so
    # the best-first tree reaches every drafted depth while its siblings interleave with the
    # path in node order (the moved rows are then the path's nodes past their slots)
    rng = np.random.default_rng(7)
    lg = logits.clone()
    for dep in range(lg.shape[0]):
        lg[dep, int(rng.integers(V))] = 16.4
    x = lg.to(torch.bfloat16).to(dev)
    root = torch.zeros(1, dtype=torch.int64, device=dev)
    tree = K.topk_tree(x, budget, root, prefix)
    n = int(tree.node_count.item()) + 1
    parents = tree.parents[:n].cpu().numpy()
    tokens = tree.verify_ids[:n].cpu().numpy()
    depth = np.zeros(n, np.int64)
    for i in range(1, n):
        depth[i] = depth[parents[i]] + 1
    target = int(np.flatnonzero(depth == depth.max())[-1])  # deepest, last in node order
    path = [target]
    while path[-1] != 0:
        path.append(int(parents[path[-1]]))
    path = path[::-1]
    post = np.zeros(n, np.int64)
    for a, b in zip(path[:-1], path[1:]):
        post[a] = tokens[b]
    child_tokens = {int(tokens[c]) for c in range(1, n) if parents[c] == target}
    t = 0
    while t in child_tokens:
        t += 1
    post[target] = t
    posterior = torch.from_numpy(post).to(dev)
    seq = prefix + n
    cache = [torch.randn((1, hkv, seq, d), device=dev).to(torch.bfloat16)
             for _ in range(2 * layers)]
    table = K.KvTable(cache)
    accepted = torch.zeros(n, dtype=torch.int64, device=dev)
    n_acc = torch.zeros(1, dtype=torch.int32, device=dev)
    nxt = torch.zeros(1, dtype=torch.int64, device=dev)

    def step():
        K.accept_compact(posterior, tree, table, prefix, accepted, n_acc, nxt, n_nodes=n)

    ms = _timed_launches(step, steps, warmup, dev)
    acc = accepted[:int(n_acc.item())].cpu().tolist()
    if acc != path:
        raise RuntimeError(f"forced path not accepted: {acc} vs {path}")
    moved = sum(1 for i, a in enumerate(acc) if a != i)
    nbytes = 2 * layers * hkv * moved * d * 2 * 2
    peaks, kind = measured_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"ms": ms, "gbs": gbs, "frac": gbs / peaks["hbm_gbs"], "peak": peaks["hbm_gbs"],
            "peak_source": kind, "bytes_per_launch": nbytes, "accepted": len(acc),
            "moved_rows_per_tensor": moved,
            "shape": f"36 layers x K/V [1, 8, {seq}, 128] bf16, forced path of {len(acc)} rows"}


def measure_compact_batched(dev, n_requests, steps, warmup, prefix=1024):
    """The batched walk + compaction (ddt_accept_compact_batched) over the request mix's trees
    (budgets of the mix, drafter logits with one lifted token per depth as in
    measure_compact), each request's posterior forced along the path to its deepest node, on
    Qwen3-8B-shaped caches (36 layers x K, V [8, prefix + budget + 1, 128] bf16, one cache per
    request).  GB/s of the algorithmic bytes (read + write of every moved row)."""
    from mdflash_b200 import kernels as K
    from mdflash_b200 import sharding as S
    layers, hkv, d = 36, 8, 128
    specs = S.request_specs(n_requests, seed=0)
    rng = np.random.default_rng(7)
    lg = torch.stack([request_logits(sp.seed) for sp in specs])
    for r in range(n_requests):
        for dep in range(lg.shape[1]):
            lg[r, dep, int(rng.integers(V))] = 16.4
    x = lg.to(torch.bfloat16).to(dev)
    trees = K.TreeBatch.allocate(dev, [sp.budget for sp in specs], DEPTHS, V)
    trees.starts.fill_(prefix)
    K.topk_tree_batched(x, trees)
    mn = trees.max_budget + 1
    post = np.zeros((n_requests, mn), np.int64)
    paths, moved = [], 0
    for r in range(n_requests):
        t = trees.tree(r)
        n = t.n_nodes
        parents = t.parents[:n].cpu().numpy()
        tokens = t.verify_ids[:n].cpu().numpy()
        depth = np.zeros(n, np.int64)
        for i in range(1, n):
            depth[i] = depth[parents[i]] + 1
        target = int(np.flatnonzero(depth == depth.max())[-1])
        path = [target]
        while path[-1] != 0:
            path.append(int(parents[path[-1]]))
        path = path[::-1]
        for a, b in zip(path[:-1], path[1:]):
            post[r, a] = tokens[b]
        post[r, target] = V  # no node carries it: the walk ends at the target
        paths.append(path)
        moved += sum(1 for i, a in enumerate(path) if a != i)
    posterior = torch.from_numpy(post).to(dev)
    tables = []
    for sp in specs:
        seq = prefix + sp.budget + 1
        tables.append(K.KvTable([torch.empty((hkv, seq, d), dtype=torch.bfloat16, device=dev)
                                 for _ in range(2 * layers)]))
    kvb = K.KvBatch(tables)
    K.accept_compact_batched(posterior, trees, kvb, [prefix] * n_requests)  # checks the windows
    pasts = torch.full((n_requests,), prefix, dtype=torch.int64, device=dev)
    out = (torch.zeros((n_requests, mn), dtype=torch.int64, device=dev),
           torch.zeros(n_requests, dtype=torch.int32, device=dev),
           torch.zeros(n_requests, dtype=torch.int64, device=dev))
    ms = _timed_launches(lambda: K.accept_compact_batched(posterior, trees, kvb, pasts, *out),
                         steps, warmup, dev)
    K.check_status(K.attention_status(dev))
    acc, nacc = out[0].cpu(), out[1].cpu()
    for r in range(n_requests):
        if acc[r, :int(nacc[r])].tolist() != paths[r]:
            raise RuntimeError(f"request {r}: forced path not accepted")
    nbytes = 2 * layers * hkv * moved * d * 2 * 2
    peaks, kind = measured_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"ms": ms, "gbs": gbs, "frac": gbs / peaks["hbm_gbs"], "peak": peaks["hbm_gbs"],
            "peak_source": kind, "bytes_per_launch": nbytes, "requests": n_requests,
            "moved_rows_per_tensor_total": moved,
            "shape": f"{n_requests} requests, 36 layers x K/V [8, {prefix} + budget + 1, 128] "
                     f"bf16, forced paths to the deepest node"}


def measure_lm_head(dev, rows, steps, warmup, hidden=QWEN3_8B["hidden"]):
    """Fused lm_head -> argmax (ddt_lm_head_argmax) at the Qwen3-8B verify shape against the
    unfused path it replaces (cuBLAS bf16 GEMM writing the logits, then ddt_argmax).  Bound:
    the weight read (V x hidden bf16) and the GEMM FLOPs, whichever is slower."""
    from mdflash_b200 import kernels as K
    g = torch.Generator(device=dev).manual_seed(0)
    h = torch.randn((rows, hidden), generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn((V, hidden), generator=g, device=dev) * hidden ** -0.5).to(torch.bfloat16)
    out = torch.empty(rows, dtype=torch.int64, device=dev)
    ms = _timed_launches(lambda: K.lm_head_argmax(h, w, out=out), steps, warmup, dev)
    K.check_status(K.attention_status(dev))
    post_unfused = torch.empty(rows, dtype=torch.int64, device=dev)
    ms_unfused = _timed_launches(lambda: K.argmax(torch.matmul(h, w.t()), out=post_unfused),
                                 steps, warmup, dev)
    agree = (out == post_unfused).float().mean().item()
    peaks, kind = measured_peaks()
    nbytes = w.numel() * 2
    flops = 2.0 * rows * hidden * V
    bound_ms = max(nbytes / (peaks["hbm_gbs"] * 1e9), flops / (peaks["bf16_tflops"] * 1e12)) * 1e3
    return {"ms": ms, "unfused_ms": ms_unfused, "speedup_vs_unfused": ms_unfused / ms,
            "tflops": flops / (ms / 1e3) / 1e12, "gbs": nbytes / (ms / 1e3) / 1e9,
            "bound_ms": bound_ms, "frac": bound_ms / ms, "peak_source": kind,
            "peak": peaks["bf16_tflops"], "posterior_agreement_vs_unfused": agree,
            "shape": f"[{rows}, {hidden}] x [{V}, {hidden}]^T bf16 -> argmax per row"}


def kernel_table(dev, args):
    steps, warmup = 20, 3
    return {
        "l2": "256 MB buffer written before every launch (L2 flushed); CUDA events per launch",
        "tree_build": measure_tree(dev, VERIFY_BUDGET, steps, warmup),
        "tree_build_batched": measure_tree_batched(dev, args.requests, steps, warmup),
        "argmax": measure_argmax(dev, VERIFY_BUDGET + 1, steps, warmup),
        "accept_compact": measure_compact(dev, VERIFY_PREFIX, VERIFY_BUDGET, steps, warmup),
        "accept_compact_batched": measure_compact_batched(dev, args.requests, steps, warmup),
        "tree_attention": measure_attn(dev, VERIFY_PREFIX, VERIFY_BUDGET, steps, warmup),
        "lm_head_argmax": measure_lm_head(dev, VERIFY_BUDGET + 1, steps, warmup),
    }


def _op_line(metric, unit, r, args, workload, bound, value_key):
    return {"metric": metric, "value": r[value_key], "unit": unit, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": workload,
                       "l2": "256 MB buffer written between launches (L2 flushed)"},
            "roofline": {"bound": bound, "achieved": r[value_key], "peak": r["peak"],
                         "unit": unit, "frac": r["frac"], "peak_source": r["peak_source"]},
            "detail": r}


def run_single(args):
    """--workload verify / attn / tree / argmax / compact on one GPU."""
    from mdflash_b200 import attention as A
    from mdflash_b200 import kernels as K
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    K._lib.load(build_if_missing=False)
    if args.workload == "verify":
        from mdflash_b200.runner import Qwen3VerifyRunner
        model = gpu_model(dev, A.register())
        with ClockSampler(_gpu_index(0)) as clocks:
            r = verify_step(args, model, Qwen3VerifyRunner(model), dev, args.steps, args.warmup,
                            args.prefix, args.budget)
        line = {"metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": 1,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic", "config": {"workload": r["workload"]},
                "roofline": r["roofline"], "detail": r, "clocks": clocks.summary()}
    elif args.workload == "attn":
        r = measure_attn(dev, args.prefix, args.budget, args.steps, args.warmup)
        line = _op_line("tree-attn TFLOP/s", "TFLOP/s", r, args, "tree attention op: " + r["shape"],
                        "tensor", "tflops")
    elif args.workload == "tree":
        r = measure_tree(dev, args.budget, args.steps, args.warmup)
        line = _op_line("tree build GB/s", "GB/s", r, args, "tree build: " + r["shape"], "hbm",
                        "gbs")
    elif args.workload == "treebatch":
        r = measure_tree_batched(dev, args.requests, args.steps, args.warmup)
        line = _op_line("batched tree build GB/s", "GB/s", r, args, "batched tree build: " +
                        r["shape"], "hbm", "gbs")
    elif args.workload == "compactbatch":
        r = measure_compact_batched(dev, args.requests, args.steps, args.warmup)
        line = _op_line("batched compaction GB/s", "GB/s", r, args,
                        "batched accept walk + KV compaction: " + r["shape"], "hbm", "gbs")
    elif args.workload == "argmax":
        r = measure_argmax(dev, args.budget + 1, args.steps, args.warmup)
        line = _op_line("argmax GB/s", "GB/s", r, args, "argmax over " + r["shape"], "hbm", "gbs")
    elif args.workload == "lmhead":
        r = measure_lm_head(dev, args.budget + 1, args.steps, args.warmup)
        line = _op_line("lm_head+argmax TFLOP/s", "TFLOP/s", r, args,
                        "fused lm_head -> argmax: " + r["shape"], "max(hbm, tensor)", "tflops")
    else:
        r = measure_compact(dev, args.prefix, args.budget, args.steps, args.warmup)
        line = _op_line("compaction GB/s", "GB/s", r, args,
                        "accept walk + KV compaction: " + r["shape"], "hbm", "gbs")
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- split-KV (cfg 5)
def run_splitkv(args):
    """Tree attention over one 131072-key prefix (Hq 32 / Hkv 8, D 128, 513 tree rows of a
    seeded random tree) whose K/V are sharded along the sequence across the GPUs: each rank
    computes the partial (O, m, l) of its shard, the partials are exchanged (NVLink peer
    stores into every rank's buffer, or --exchange nccl: one all-gather) and merged; the last
    rank owns the tree keys and compacts the accepted path inside its shard.  The exchange and merge are timed apart from the shard's
    attention (CUDA events on the step stream)."""
    import torch.distributed as dist

    from mdflash_b200 import kernels as K
    from mdflash_b200 import sharding as S

    world, rank, local, dev = _dist_setup()
    K._lib.load(build_if_missing=False)
    P, B = args.prefix, args.budget
    n = B + 1
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import inputs as gin
    parents = gin.random_tree(n, 5)
    bits = torch.from_numpy(anc_bits_host(parents).view(np.int32)).to(dev)
    kb, ke = S.shard_range(P, n, world, rank)
    g = torch.Generator(device=dev).manual_seed(11)
    sc = 1.0 / math.sqrt(128)
    q = (torch.randn((n, 32, 128), generator=g, device=dev) * sc).to(torch.bfloat16)
    gk = torch.Generator(device=dev).manual_seed(100 + rank)
    k = (torch.randn((8, ke - kb, 128), generator=gk, device=dev) * sc).to(torch.bfloat16)
    v = torch.randn((8, ke - kb, 128), generator=gk, device=dev).to(torch.bfloat16)
    out = torch.empty((n, 32, 128), dtype=torch.bfloat16, device=dev)
    owner = rank == S.owner_rank(world)
    depth = np.zeros(n, np.int64)
    for i in range(1, n):
        depth[i] = depth[parents[i]] + 1
    path = [int(np.argmax(depth))]
    while path[-1] != 0:
        path.append(int(parents[path[-1]]))
    keep = torch.tensor(path[::-1], dtype=torch.int64, device=dev)
    table = K.KvTable([k, v])
    xchg = S.PeerExchange(n, 32, dev) if args.exchange == "peer" else None

    def step(events=None):
        if events:
            events[0].record()
        if xchg is not None:  # the merge of the shard's splits stores into every rank's buffer
            xchg.attend_push(q, k, v, kb, ke, bits, P)
        else:
            o, m, l = K.tree_attention_partial_merged(q, k, v, kb, ke, bits, P)
        if events:
            events[1].record()
        if xchg is not None:
            xchg.merge(out)
        else:
            og, mg, lg = S.gather_partials(o, m, l)
            K.attn_merge(og, mg, lg, n, 32, out=out)
        if events:
            events[2].record()
        if owner:  # compaction of the accepted path on the rank holding the tree keys
            S.compact_owner_shard(keep, table, (kb, ke), P)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    K.check_status(K.attention_status(dev))
    parts = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        step(evs)
        parts.append(evs)
    b.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    K.check_status(K.attention_status(dev))
    shard_ms = float(np.mean([e[0].elapsed_time(e[1]) for e in parts]))
    xchg_ms = float(np.mean([e[1].elapsed_time(e[2]) for e in parts]))
    t = torch.tensor([a.elapsed_time(b) / args.steps, shard_ms, xchg_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, shard_ms, xchg_ms = t.tolist()
    flops = attn_flops(parents, P)
    peaks, kind = measured_peaks()
    tflops = flops / (ms / 1e3) / 1e12
    link_bytes = (world - 1) * n * 32 * (128 + 2) * 4  # partials each rank receives
    line = {
        "metric": "tree-attn TFLOP/s", "value": tflops, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"split-KV tree attention: prefix {P} sharded over {world} GPUs, "
                               f"{n} tree rows, Hq 32 / Hkv 8, D 128; compaction of a "
                               f"{len(path)}-row path on the owner shard",
                   "exchange": ("the shard's split merge stores the fp32 (O, m, l) partial "
                                "into every rank's buffer over NVLink (ddt_tree_attn_partial_push)"
                                "; counter wait and merge (ddt_peer_merge)" if xchg is not None else
                                "NCCL all-gather of fp32 (O, m, l) partials + ddt_attn_merge"),
                   "partial_bytes_received_per_rank": link_bytes},
        "split": {"shard_attention_ms": shard_ms, "exchange_and_merge_ms": xchg_ms,
                  "note": "max over ranks of each part; the rest of ms_per_step is the owner's "
                          "compaction and host launch gaps"},
        "roofline": {"bound": "tensor", "achieved": tflops / world, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s per GPU", "frac": tflops / world / peaks["bf16_tflops"],
                     "peak_source": f"{kind} bf16 burst", "flops_per_step": flops},
    }
    if xchg is not None:
        xchg.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "requests":
        return run_requests(args)
    if args.workload == "splitkv":
        return run_splitkv(args)
    return run_single(args)


if __name__ == "__main__":
    main()
