#!/usr/bin/env python
"""Benchmark of the DDTree verify step on B200.

Workload (one "step"): the single-GPU verify step of a random-init Qwen3-8B-shaped target
(36 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128, MLP 12288, vocab 151936, bf16)
over a prefix of 8192 uniform-random tokens, with per-depth drafter logits for block
length 16 (15 depths, seeded N(0,1)*3) driving a 256-node best-first tree (257 rows with
the root): tree build -> tree-attention verify forward -> greedy posterior -> accept walk
-> KV compaction.  Metric: verified + accepted tokens per second (257 verified rows plus
the committed path per step), summed over GPUs.

  value      inputs resident in HBM; K steps back to back, CUDA events on the step stream
  e2e        the same through the public API with host buffers: each step copies the
             draft logits + root token from pinned host memory and reads the result back
  roofline   the tree-attention launches are bracketed by CUDA events inside the timed
             region; achieved TFLOP/s = algorithmic FLOPs per launch / mean launch time
  cpu_baseline  the CPU oracle path (C tree build, torch CPU Qwen3 layers with the
             reference's SDPA + additive mask, argmax, walk, compaction) on a bounded
             sample: 2 of the 36 layers timed per layer and scaled to 36

--gpus N (under torchrun): every rank verifies its own request (request data
parallelism, no data-path collective); the step time is the max over ranks.
--impl reference: the CPU oracle path alone on this host's cores (rank 0 only).
"""
from __future__ import annotations

import argparse
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
METRIC = "verified+accepted tokens/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["verify", "attn", "tree", "argmax", "compact",
                                           "requests", "splitkv"],
                    default="verify",
                    help="verify: the single-request verify step (default); attn / tree / argmax "
                         "/ compact: one op alone; requests: 64 requests sharded over the GPUs; "
                         "splitkv: attention over a prefix sharded along the sequence")
    ap.add_argument("--prefix", type=int, default=None,
                    help="prefix length (default 8192; 131072 for --workload splitkv)")
    ap.add_argument("--budget", type=int, default=None,
                    help="tree budget (default 256; 512 for --workload splitkv)")
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--cpu-sample-layers", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--fused", type=int, default=1,
                    help="1: verify forward through the fused Qwen3 runner (default); 0: through "
                         "transformers' Qwen3 with the ddtree_tree attention plug-in")
    args = ap.parse_args()
    long_ctx = args.workload == "splitkv"
    if args.prefix is None:
        args.prefix = 131072 if long_ctx else 8192
    if args.budget is None:
        args.budget = 512 if long_ctx else 256
    return args


def qwen3_config(attn: str, layers: int | None = None):
    from transformers import Qwen3Config
    s = QWEN3_8B
    return Qwen3Config(vocab_size=s["vocab"], hidden_size=s["hidden"], intermediate_size=s["mlp"],
                       num_hidden_layers=layers or s["layers"], num_attention_heads=s["heads"],
                       num_key_value_heads=s["kv_heads"], head_dim=s["head_dim"],
                       rope_theta=s["rope_theta"], max_position_embeddings=40960, rms_norm_eps=1e-6,
                       tie_word_embeddings=False, attn_implementation=attn)


def request_inputs(rank: int, prefix: int):
    rng = np.random.default_rng(1000 + rank)
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


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic():
    """DRAM bytes per tree-attention launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "tree_attn_traffic.json")
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
                 "-lms", "20", "-i", str(self.gpu_index)], stdout=self.tmp,
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


# ------------------------------------------------------------------ CPU oracle path
def cpu_verify_sample(sample_layers: int, prefix: int, budget: int, steps: int, warmup: int):
    """The reference's verify step on the host cores through the CPU oracle: C tree build,
    compile (additive mask), a Qwen3-8B-shaped forward of `sample_layers` decoder layers
    with SDPA + mask (fp32), argmax, walk and compaction of `sample_layers` layers.  The
    per-layer costs are timed with hooks and scaled to the 36 layers of the model."""
    import oracle
    from transformers import DynamicCache, Qwen3ForCausalLM
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    with torch.inference_mode():
        model = Qwen3ForCausalLM(qwen3_config("sdpa", sample_layers)).eval().float()
    ids, logits = request_inputs(0, prefix)
    logits = logits.to(torch.bfloat16)  # the drafter logits the GPU arm sees
    n_cap = budget + 1
    g = torch.Generator().manual_seed(0)
    kv = [(torch.randn((1, 8, prefix, 128), generator=g) * 0.5,
           torch.randn((1, 8, prefix, 128), generator=g) * 0.5) for _ in range(sample_layers)]
    layer_times: list[float] = []
    starts: dict[int, float] = {}

    def pre(mod, args, kwargs):
        starts[id(mod)] = time.perf_counter()

    def post(mod, args, kwargs, out):
        layer_times.append(time.perf_counter() - starts[id(mod)])

    for layer in model.model.layers:
        layer.register_forward_pre_hook(pre, with_kwargs=True)
        layer.register_forward_hook(post, with_kwargs=True)
    per_step = []
    n_acc = 1
    root = int(ids[0, -1])
    for it in range(warmup + steps):
        cache = DynamicCache()
        for li, (k, v) in enumerate(kv):
            cache.update(k.clone(), v.clone(), li)
        layer_times.clear()
        t0 = time.perf_counter()
        node_ids, depths, parents, child_maps, vis, _ = oracle.build_ddtree_tree(logits, budget)
        t1 = time.perf_counter()
        vib = torch.empty((1, n_cap), dtype=torch.long)
        vpb = torch.empty((1, n_cap), dtype=torch.long)
        amb = torch.zeros((1, 1, n_cap, prefix + n_cap), dtype=torch.float32)
        tvb = torch.empty((n_cap, n_cap), dtype=torch.bool)
        vi, vp, am, _, n = oracle.compile_ddtree_tree(root, prefix, node_ids, depths, vis, prefix,
                                                      torch.float32, None, vib, vpb, amb, tvb, 0, 0)
        with torch.inference_mode():
            t2 = time.perf_counter()
            out = model(vi, position_ids=vp, attention_mask=am, past_key_values=cache,
                        use_cache=True)
            t3 = time.perf_counter()
            post_tokens = oracle.argmax(out.logits[0])
            acc, nxt = oracle.follow_verified_tree(child_maps, post_tokens)
            layers_np = [(l.keys.numpy(), l.values.numpy()) for l in cache.layers]
            oracle.compact_dynamic_cache(layers_np, prefix, acc)
            t4 = time.perf_counter()
        fwd_layers = sum(layer_times)
        fwd_other = (t3 - t2) - fwd_layers
        commit = t4 - t3
        step = ((t1 - t0) + (t2 - t1) + fwd_other + fwd_layers * 36 / sample_layers +
                commit * 36 / sample_layers)  # compaction also covers every layer
        n_acc = len(acc)
        if it >= warmup:
            per_step.append(step)
    t = float(np.mean(per_step))
    return {"seconds_per_step": t, "tokens_per_step": n + n_acc, "threads": threads,
            "sample": f"{sample_layers} of 36 decoder layers timed (forward hooks) and scaled to "
                      f"36; tree build, compile, embed, lm_head and argmax at full size; "
                      f"prefix {prefix} K/V random fp32; {steps} steps after {warmup} warm-up"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    r = cpu_verify_sample(args.cpu_sample_layers, args.prefix, args.budget, args.steps,
                          args.warmup)
    value = r["tokens_per_step"] / r["seconds_per_step"]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["seconds_per_step"] * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": r["threads"],
                         "kind": "port", "sample": r["sample"]},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args, n):
    return {"workload": f"Qwen3-8B-shaped verify step: 36 layers, prefix {args.prefix}, "
                        f"{args.budget}-node best-first tree (block 16 -> 15 depths), bf16",
            "model": "Qwen3-8B shape, random init", "global_batch": n,
            "seq_len": args.prefix, "tree_nodes": args.budget + 1,
            "parallelism": f"request-dp{n}",
            "l2": "inputs larger than L2: 16 GB of weights and 1.2 GB of KV streamed per step"}


# ------------------------------------------------------------------------ our arm
def run_ours(args):
    import torch.distributed as dist
    from transformers import Qwen3ForCausalLM

    from mdflash_b200 import attention as A
    from mdflash_b200 import kernels as K
    from mdflash_b200.cache import TreeKVCache
    from mdflash_b200.verifier import CapturedStep, TreeVerifier

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    K._lib.load(build_if_missing=False)
    attn = A.register()
    torch.manual_seed(rank)
    prev_dtype = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev), torch.inference_mode():
        model = Qwen3ForCausalLM(qwen3_config(attn)).eval()
    torch.set_default_dtype(prev_dtype)
    ids, logits = request_inputs(rank, args.prefix)
    P, B = args.prefix, args.budget
    cache = TreeKVCache(QWEN3_8B["layers"], P + B + 1 + 64).allocate(
        QWEN3_8B["kv_heads"], QWEN3_8B["head_dim"], torch.bfloat16, dev)
    verifier = TreeVerifier(model, cache, B, DEPTHS, V, dev, fused=args.fused)
    with torch.inference_mode():
        if verifier.runner is not None:  # causal prefill on the same kernels
            out_logits = verifier.runner.forward(ids[0].to(dev), torch.arange(P, device=dev),
                                                 cache, 0, None, causal=True)
            root_dev = K.argmax(out_logits[-1:]).view(1).clone()
            del out_logits
        else:
            out = model(ids.to(dev), position_ids=torch.arange(P, device=dev)[None],
                        past_key_values=cache, use_cache=True, logits_to_keep=1)
            root_dev = K.argmax(out.logits[0, -1:]).view(1).clone()
            del out
    draft_dev = logits.to(torch.bfloat16).to(dev)
    n_nodes = 1 + K.expected_node_count(DEPTHS, V, B)
    for _ in range(args.warmup):  # eager steps: allocations, kernel attributes, TMA encode
        verifier.step(draft_dev, root_dev, P)
        cache.crop(P)  # every step verifies the same prefix (the commit is undone)
    # the whole step (tree build, 36-layer forward, argmax, walk + compaction) as one graph
    cap = CapturedStep(verifier, P, warmup=1, time_attention=True)
    cap.draft_logits.copy_(draft_dev)
    cap.root_token.copy_(root_dev)
    for _ in range(args.warmup):
        cap.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- device-resident timing (value + attention roofline) ----
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_index = int(visible.split(",")[local]) if visible else local
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_index) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.nvtx.range_push("timed")
        ev0.record()
        for _ in range(args.steps):
            res = cap.replay()
        ev1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    launches = cap.launches_per_replay * args.steps
    attn_ms = cap.attention_ms()  # the last replay of the timed region
    ms = ev0.elapsed_time(ev1) / args.steps
    n_acc = int(res.n_accepted.item())
    depths = verifier.tree.node_depths[:n_nodes - 1].cpu()
    ms_t = torch.tensor([ms], device=dev)
    acc_t = torch.tensor([float(n_nodes + n_acc)], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        dist.all_reduce(acc_t, op=dist.ReduceOp.SUM)
        dist.barrier()
    ms_max = ms_t.item()
    tokens_all = acc_t.item()
    value = tokens_all / (ms_max / 1e3)

    # ---- end to end through the public API with host buffers ----
    draft_host = logits.to(torch.bfloat16).pin_memory()
    root_host = torch.zeros(1, dtype=torch.int64).pin_memory()
    root_host.copy_(root_dev.cpu())
    result_host = torch.zeros(2 + n_nodes, dtype=torch.int64).pin_memory()

    def e2e_step():
        cap.draft_logits.copy_(draft_host, non_blocking=True)
        cap.root_token.copy_(root_host, non_blocking=True)
        r = cap.replay()
        packed = torch.cat([r.n_accepted.to(torch.int64), r.next_token, r.accepted[:n_nodes]])
        result_host.copy_(packed, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return int(result_host[0])

    for _ in range(args.warmup):
        e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    ks = [e2e_step() for _ in range(args.steps)]
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    e2e_tok = torch.tensor([float(sum(n_nodes + k for k in ks) / args.steps)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(e2e_tok, op=dist.ReduceOp.SUM)
    e2e_value = e2e_tok.item() / (e2e_ms.item() / 1e3)
    h2d = draft_host.numel() * draft_host.element_size() + root_host.numel() * 8
    d2h = result_host.numel() * 8

    # ---- roofline of the dominant kernel (tree attention, one launch per layer) ----
    peaks, peak_kind = measured_peaks()
    flops = tree_flops(depths, P, QWEN3_8B["heads"], QWEN3_8B["head_dim"])
    attn_mean_ms = float(np.mean(attn_ms)) if attn_ms else float("nan")
    achieved = flops / (attn_mean_ms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    traffic = profile_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded uniform prefix tokens, N(0,1)*3 drafter logits, random-init "
                "Qwen3-8B-shaped weights",
        "config": workload_config(args, world),
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms.item()},
        "roofline": {"kernel": "ddt_tree_attn (+ split merge), one launch per layer",
                     "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak,
                     "peak_source": f"{peak_kind} bf16 sustained (MEASURED_PEAKS.json)",
                     "flops_per_launch": flops, "launch_ms": attn_mean_ms,
                     "launches_timed": len(attn_ms),
                     "traffic": traffic.get("bytes_per_launch") if traffic else None},
        "gpu_launches": launches,
        "launches_per_step": launches / args.steps,
        "execution": "each step is one CUDA-graph replay of the full verify step (tree build, "
                     "36-layer forward, argmax, accept walk + compaction) at prefix length "
                     f"{P}; eager warm-up steps precede the capture; forward: "
                     + ("fused Qwen3 runner (cuBLAS GEMMs + fused norm/rope/silu kernels)"
                        if args.fused else "transformers Qwen3 + ddtree_tree attention"),
        "accepted_per_step": n_acc, "verified_per_step": n_nodes,
        "attention_share": (attn_mean_ms * QWEN3_8B["layers"]) / ms,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_verify_sample(args.cpu_sample_layers, args.prefix, args.budget, 1, 1)
        line["cpu_baseline"] = {"value": r["tokens_per_step"] / r["seconds_per_step"],
                                "unit": "tokens/s", "cores": r["threads"], "kind": "port",
                                "sample": r["sample"]}
    line["clocks"] = clocks.summary()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------- op-level attention
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


def run_attn(args):
    from mdflash_b200 import kernels as K
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q, k, v, parents = attn_inputs(args.prefix, args.budget)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    bits = torch.from_numpy(anc_bits_host(parents).view(np.int32)).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > 126 MB L2
    out = K.tree_attention(qd, kd, vd, bits, args.prefix)
    for _ in range(args.warmup):
        K.tree_attention(qd, kd, vd, bits, args.prefix, out=out)
    torch.cuda.synchronize()
    times = []
    torch.cuda.nvtx.range_push("timed")
    for _ in range(args.steps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        K.tree_attention(qd, kd, vd, bits, args.prefix, out=out)
        b.record()
        times.append((a, b))
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = float(np.mean([a.elapsed_time(b) for a, b in times]))
    flops = attn_flops(parents, args.prefix)
    peaks, kind = measured_peaks()
    peak = float(peaks["bf16_tflops"])
    tflops = flops / (ms / 1e3) / 1e12
    kv_bytes = 2 * 8 * (args.prefix + args.budget + 1) * 128 * 2
    print(json.dumps({
        "metric": "tree-attn TFLOP/s", "value": tflops, "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"tree attention op: Hq 32 / Hkv 8, D 128, prefix {args.prefix}, "
                               f"{args.budget + 1} tree rows (random tree, Geometric(0.5))",
                   "l2": "256 MB buffer written between launches (L2 flushed)",
                   "kv_splits": K.attn_splits(args.budget + 1, 32, 8, args.prefix)},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                     "frac": tflops / peak, "peak_source": f"{kind} bf16 burst",
                     "flops_per_launch": flops, "kv_bytes": kv_bytes},
    }), flush=True)


def run_tree(args):
    """Tree construction op alone: [15, 151936] bf16 drafter logits -> tree (top-k, heap,
    bitmasks, verify ids / positions).  Reports GB/s of the algorithmic bytes (one read of
    the logits) over the launch time, L2 flushed between launches."""
    from mdflash_b200 import kernels as K
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _, logits = request_inputs(0, 16)
    x = logits.to(torch.bfloat16).to(dev)
    root = torch.zeros(1, dtype=torch.int64, device=dev)
    tree = K.topk_tree(x, args.budget, root, args.prefix)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        K.topk_tree(x, args.budget, root, args.prefix, out=tree)
    torch.cuda.synchronize()
    times = []
    torch.cuda.nvtx.range_push("timed")
    for _ in range(args.steps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        K.topk_tree(x, args.budget, root, args.prefix, out=tree)
        b.record()
        times.append((a, b))
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = float(np.mean([a.elapsed_time(b) for a, b in times]))
    nbytes = x.numel() * x.element_size()
    peaks, kind = measured_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "tree build GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"tree build: 15 x {V} bf16 logits, budget {args.budget}",
                   "l2": "256 MB buffer written between launches (L2 flushed)"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "peak_source": kind},
        "node_count": int(tree.node_count.item()),
    }), flush=True)


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


def run_argmax(args):
    """Greedy posterior (model/utils.py:28-30 at T=0) alone: argmax over [N, 151936] bf16
    verify logits, N = budget + 1.  GB/s of the algorithmic bytes (one read of the logits)."""
    from mdflash_b200 import kernels as K
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = args.budget + 1
    g = torch.Generator(device=dev).manual_seed(0)
    logits = torch.randn((n, V), generator=g, device=dev).mul_(3).to(torch.bfloat16)
    out = torch.empty(n, dtype=torch.int64, device=dev)
    ms = _timed_launches(lambda: K.argmax(logits, out=out), args.steps, args.warmup, dev)
    nbytes = logits.numel() * logits.element_size()
    peaks, kind = measured_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "argmax GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"argmax over [{n}, {V}] bf16 verify logits (N(0,1)*3)",
                   "l2": "256 MB buffer written between launches (L2 flushed)"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "peak_source": kind,
                     "bytes_per_launch": nbytes},
    }), flush=True)


def run_compact(args):
    """Accept walk + KV compaction alone on the Qwen3-8B cache shape (36 layers x K, V
    [1, 8, P + N, 128] bf16) with a forced accepted path: the posterior follows the tree
    from the root to its deepest node (the drafter logits make the tree reach all 15
    depths), so a 16-row path is accepted and each layer's K and V move one row per
    accepted node not already in place.  GB/s of the algorithmic
    bytes (read + write of every moved row) over the launch time."""
    from mdflash_b200 import kernels as K
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    layers, hkv, d = 36, 8, 128
    _, logits = request_inputs(0, 16)
    # one token per depth lifted to about the log-sum-exp of the rest (log-prob ~ -0.7), so
    # the best-first tree reaches every drafted depth while its siblings interleave with the
    # path in node order (the moved rows are then the path's nodes past their slots)
    rng = np.random.default_rng(7)
    lg = logits.clone()
    for dep in range(lg.shape[0]):
        lg[dep, int(rng.integers(V))] = 16.4
    x = lg.to(torch.bfloat16).to(dev)
    root = torch.zeros(1, dtype=torch.int64, device=dev)
    tree = K.topk_tree(x, args.budget, root, args.prefix)
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
    seq = args.prefix + n
    cache = [torch.randn((1, hkv, seq, d), device=dev).to(torch.bfloat16)
             for _ in range(2 * layers)]
    table = K.KvTable(cache)
    accepted = torch.zeros(n, dtype=torch.int64, device=dev)
    n_acc = torch.zeros(1, dtype=torch.int32, device=dev)
    nxt = torch.zeros(1, dtype=torch.int64, device=dev)

    def step():
        K.accept_compact(posterior, tree, table, args.prefix, accepted, n_acc, nxt, n_nodes=n)

    ms = _timed_launches(step, args.steps, args.warmup, dev)
    acc = accepted[:int(n_acc.item())].cpu().tolist()
    assert acc == path, (acc, path)
    moved = sum(1 for i, a in enumerate(acc) if a != i)
    nbytes = 2 * layers * hkv * moved * d * 2 * 2
    peaks, kind = measured_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "compaction GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"accept walk + KV compaction, Qwen3-8B cache (36 layers x K/V "
                               f"[1, 8, {seq}, 128] bf16), forced path of {len(acc)} accepted "
                               f"rows, {moved} moved per tensor",
                   "l2": "256 MB buffer written between launches (L2 flushed)"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "peak_source": kind,
                     "bytes_per_launch": nbytes},
        "accepted": len(acc),
    }), flush=True)


# ------------------------------------------------------------- multi-GPU workloads
def _dist_setup():
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    return world, rank, dev


def run_requests(args):
    """64 independent requests (prefix log-uniform 1k..32k, budget in {64,128,256,512},
    per-request drafter seeds) assigned to ranks by longest-processing-time; each rank
    verifies its requests one after another (one CUDA-graph replay each), then the result
    records are all-gathered.  Prefix K/V are random bf16 (the verify work does not depend
    on their values); the step for each request is the full verify step."""
    import torch.distributed as dist
    from transformers import Qwen3ForCausalLM

    from mdflash_b200 import attention as A
    from mdflash_b200 import kernels as K
    from mdflash_b200 import sharding as S
    from mdflash_b200.cache import TreeKVCache
    from mdflash_b200.runner import Qwen3VerifyRunner
    from mdflash_b200.verifier import CapturedStep, TreeVerifier

    world, rank, dev = _dist_setup()
    K._lib.load(build_if_missing=False)
    attn = A.register()
    torch.manual_seed(0)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev), torch.inference_mode():
        model = Qwen3ForCausalLM(qwen3_config(attn)).eval()
    torch.set_default_dtype(prev)
    runner = Qwen3VerifyRunner(model)
    specs = S.request_specs(args.requests, seed=0)
    mine = S.assign_requests([S.request_cost(s) for s in specs], world)[rank]
    pool = torch.cuda.graph_pool_handle()
    caps = []
    g = torch.Generator(device=dev).manual_seed(rank)
    for i in mine:
        sp = specs[i]
        cache = TreeKVCache(QWEN3_8B["layers"], sp.prefix + sp.budget + 1 + 64).allocate(
            QWEN3_8B["kv_heads"], QWEN3_8B["head_dim"], torch.bfloat16, dev)
        for layer in cache.layers:
            layer.k_buf.normal_(0.0, 1.0, generator=g)
            layer.v_buf.normal_(0.0, 1.0, generator=g)
            layer.length = sp.prefix
            layer.keys = layer.k_buf[..., :sp.prefix, :]
            layer.values = layer.v_buf[..., :sp.prefix, :]
        ver = TreeVerifier(model, cache, sp.budget, DEPTHS, V, dev, runner=runner)
        cap = CapturedStep(ver, sp.prefix, warmup=1, pool=pool)
        rng = np.random.default_rng(sp.seed)
        cap.draft_logits.copy_(torch.from_numpy(
            rng.standard_normal((DEPTHS, V)).astype(np.float32) * np.float32(3.0)).to(torch.bfloat16))
        cap.root_token.fill_(int(rng.integers(0, V)))
        caps.append((sp, cap))
    for _ in range(args.warmup):
        for _, cap in caps:
            cap.replay()
    local = torch.full((len(caps), S.RECORD_LEN), -1, dtype=torch.int64, device=dev)
    for j, (sp, cap) in enumerate(caps):
        local[j, :3] = torch.tensor([sp.index, rank, cap.result.n_nodes])
        local[j, 5] = 0
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    allrec = None
    for _ in range(args.steps):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev0.record()
        for j, (sp, cap) in enumerate(caps):
            r = cap.replay()
            # record on the device: [index, rank, n_nodes | n_accepted, next | 0 | path]
            local[j, 3] = r.n_accepted[0]
            local[j, 4] = r.next_token[0]
            m = min(S.MAX_PATH, r.n_nodes)
            local[j, 6:6 + m] = r.accepted[:m]
        allrec = S.gather_results(local)
        ev1.record()
        torch.cuda.synchronize()
        t = torch.tensor([ev0.elapsed_time(ev1)], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times.append(t.item())
    ms = float(np.mean(times))
    host = allrec.cpu()
    tokens = int((host[:, 2] + host[:, 3]).sum())
    value = tokens / (ms / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded request mix, random prefix K/V, N(0,1)*3 drafter logits, "
                "random-init Qwen3-8B-shaped weights",
        "config": {"workload": f"{args.requests} requests, prefix log-uniform 1k-32k, budget "
                               "{64,128,256,512}, Qwen3-8B shape, one verify step each",
                   "parallelism": f"request-dp{world} (longest-processing-time assignment)",
                   "requests_per_rank": [len(x) for x in S.assign_requests(
                       [S.request_cost(s) for s in specs], world)],
                   "step": "every request's verify step once + all-gather of result records"},
        "tokens_per_step": tokens,
    }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_splitkv(args):
    """Tree attention over one 131072-key prefix (Hq 32 / Hkv 8, D 128, 513 tree rows of a
    seeded random tree) whose K/V are sharded along the sequence across the GPUs: each rank
    computes the partial (O, m, l) of its shard, one NCCL all-gather exchanges them and
    ddt_attn_merge combines them (the last rank also holds the tree rows)."""
    import torch.distributed as dist

    from mdflash_b200 import kernels as K
    from mdflash_b200 import sharding as S

    world, rank, dev = _dist_setup()
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
    for _ in range(args.warmup):
        S.splitkv_attention(q, k, v, kb, ke, bits, P, out=out)
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        S.splitkv_attention(q, k, v, kb, ke, bits, P, out=out)
        b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b)], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times.append(t.item())
    ms = float(np.mean(times))
    flops = attn_flops(parents, P)
    peaks, kind = measured_peaks()
    tflops = flops / (ms / 1e3) / 1e12
    link_bytes = (world - 1) * n * 32 * (128 + 2) * 4  # partials each rank receives
    line = {
        "metric": "tree-attn TFLOP/s", "value": tflops, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"split-KV tree attention: prefix {P} sharded over {world} GPUs, "
                               f"{n} tree rows, Hq 32 / Hkv 8, D 128",
                   "exchange": "NCCL all-gather of fp32 (O, m, l) partials + ddt_attn_merge",
                   "partial_bytes_received_per_rank": link_bytes},
        "roofline": {"bound": "tensor", "achieved": tflops / world, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s per GPU", "frac": tflops / world / peaks["bf16_tflops"],
                     "peak_source": f"{kind} bf16 burst", "flops_per_step": flops},
    }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.workload == "requests":
        return run_requests(args)
    if args.workload == "splitkv":
        return run_splitkv(args)
    if args.workload == "attn":
        run_attn(args)
    elif args.workload == "tree":
        run_tree(args)
    elif args.workload == "argmax":
        run_argmax(args)
    elif args.workload == "compact":
        run_compact(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
