"""The verify step with its prefix length in device memory, so that one CUDA graph serves
every round of a decode loop (the reference's loop, ddtree.py:417-506, advances its prefix
by the accepted length every round; the host-side prefix length of ddt_tree_attn would need
a new graph per round).

* ddt_tree_attn_device_past at a live length against the fp32 reference at that length.
  K / V rows after the live window hold large values: a mask that let them through would
  move the output far beyond the bf16 tolerance.  One recorded launch, replayed at several
  live lengths, gives bit-for-bit what eager launches give.
* A live length outside [0, planned] sets the status bit that check_status reports; the
  launch stays in bounds and the next launch is correct.
* ddt_qk_norm_rope_cache_table_device_past writes bit-for-bit what the host-length form
  writes, and nothing for an out-of-range length.
* A decode loop whose steps replay ONE CapturedStep(max_start=...) against the eager step at
  the host prefix length, round by round: the same tree, posterior, accepted path and next
  token.
"""
import math

import numpy as np
import pytest
import torch

import inputs as gin
import oracle
from mdflash_b200 import _lib
from mdflash_b200 import kernels as K
from mdflash_b200._lib import DDTreeError, check
from parity_util import elem_rel_err

pytestmark = pytest.mark.gpu
ATTN_TOL = 2e-2


def _rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)).item()


def _inputs(hq, hkv, max_past, n, seed, device):
    g = torch.Generator().manual_seed(seed)
    d = 128
    sc = 1.0 / math.sqrt(d)
    q = (torch.randn((hq, n, d), generator=g) * sc).to(torch.bfloat16)
    k = (torch.randn((hkv, max_past + n, d), generator=g) * sc).to(torch.bfloat16)
    v = (torch.randn((hkv, max_past + n, d), generator=g) * sc).to(torch.bfloat16)
    parents = gin.random_tree(n, seed + 10)
    bits = torch.from_numpy(oracle.ancestor_bits(parents).view(np.int32)).to(device)
    return q, k, v, parents, bits


def _plant_after(k, v, live, n):
    """Large finite values in every row after the live window [0, live + n)."""
    k = k.clone()
    v = v.clone()
    k[:, live + n:] = 4.0
    v[:, live + n:] = 1000.0
    return k, v


@pytest.mark.parametrize("hq,hkv,max_past,n,lives,causal", [
    (32, 8, 8192, 257, [8192, 8191, 5000, 128, 0], False),   # Qwen3-8B verify shape, balanced
    (32, 8, 40000, 65, [40000, 33001], False),               # K / V beyond L2: uniform splits
    (16, 8, 700, 33, [700, 100], True),                      # causal mask (prefill form)
    (8, 8, 300, 100, [300, 17], False),                      # group 1
])
def test_tree_attention_device_past(cuda_device, hq, hkv, max_past, n, lives, causal):
    q, k, v, parents, bits = _inputs(hq, hkv, max_past, n, max_past + n, cuda_device)
    vis = oracle.visibility(parents)
    qd = q.transpose(0, 1).contiguous().to(cuda_device)
    past_dev = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    kd = k.to(cuda_device)
    vd = v.to(cuda_device)
    eager = {}
    for live in lives:
        kp, vp = _plant_after(kd, vd, live, n)
        past_dev.fill_(live)
        out = K.tree_attention(qd, kp, vp, None if causal else bits, max_past, causal=causal,
                               status=status, past_dev=past_dev)
        torch.cuda.synchronize()
        K.check_status(status, "ddt_tree_attn_device_past")
        ref = oracle.tree_attention(q.float(), k[:, :live + n].float(), v[:, :live + n].float(),
                                    None if causal else vis, live, causal=causal)
        err, eerr = _rel_err(out.cpu(), ref), elem_rel_err(out.cpu(), ref)
        print(f"[device past] max {max_past} live {live}: rel {err:.2e}, elem {eerr:.2e}")
        assert err <= ATTN_TOL and eerr <= ATTN_TOL
        eager[live] = (out.clone(), kp, vp)
    # one recorded launch replayed at every live length: bit-for-bit the eager outputs
    kbuf, vbuf = kd.clone(), vd.clone()
    out = torch.empty_like(eager[lives[0]][0])
    K.tree_attention(qd, kbuf, vbuf, None if causal else bits, max_past, causal=causal,
                     status=status, past_dev=past_dev, out=out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        K.tree_attention(qd, kbuf, vbuf, None if causal else bits, max_past, causal=causal,
                         status=status, past_dev=past_dev, out=out)
    for live in reversed(lives):
        ref_out, kp, vp = eager[live]
        kbuf.copy_(kp)
        vbuf.copy_(vp)
        past_dev.fill_(live)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out), live
    K.check_status(status, "ddt_tree_attn_device_past (graph)")


def test_tree_attention_device_past_out_of_range(cuda_device):
    """A live length outside [0, planned] is reported (status bit 4 -> DDTreeError) and the
    launch runs at the planned length, in bounds; the next launch is correct."""
    hq, hkv, max_past, n = 32, 8, 1024, 65
    q, k, v, parents, bits = _inputs(hq, hkv, max_past, n, 5, cuda_device)
    qd = q.transpose(0, 1).contiguous().to(cuda_device)
    kd, vd = k.to(cuda_device), v.to(cuda_device)
    past_dev = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for bad in (max_past + 1, -1, 1 << 40):
        past_dev.fill_(bad)
        K.tree_attention(qd, kd, vd, bits, max_past, status=status, past_dev=past_dev)
        torch.cuda.synchronize()
        assert int(status.item()) == K.STATUS_PAST_RANGE
        with pytest.raises(DDTreeError, match="prefix length out of range"):
            K.check_status(status)
        assert int(status.item()) == 0
    past_dev.fill_(600)
    out = K.tree_attention(qd, kd, vd, bits, max_past, status=status, past_dev=past_dev)
    torch.cuda.synchronize()
    K.check_status(status)
    ref = oracle.tree_attention(q.float(), k[:, :600 + n].float(), v[:, :600 + n].float(),
                                oracle.visibility(parents), 600)
    assert _rel_err(out.cpu(), ref) <= ATTN_TOL
    # the wrapper's own checks
    with pytest.raises(ValueError):
        K.tree_attention(qd, kd, vd, bits, max_past, past_dev=past_dev.to(torch.int32))
    with pytest.raises(ValueError):
        K.tree_attention(qd, kd, vd, None, max_past, unmasked=True, past_dev=past_dev)


def test_qk_norm_rope_cache_device_past(cuda_device):
    """The device-length cache write equals the host-length one bit for bit (q and the K / V
    rows), leaves every other row alone, and writes nothing for an out-of-range length."""
    n, hq, hkv, d, cap = 33, 16, 8, 128, 700
    g = torch.Generator(device=cuda_device).manual_seed(11)
    qkv = torch.randn((n, (hq + 2 * hkv) * d), generator=g, device=cuda_device).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(d, generator=g, device=cuda_device)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(d, generator=g, device=cuda_device)).to(torch.bfloat16)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, d, 2, device=cuda_device).float() / d))
    lib = _lib.load()
    st = torch.cuda.current_stream(cuda_device).cuda_stream
    max_past = cap - n
    for live in (0, 250, max_past):
        pos = torch.arange(live, live + n, device=cuda_device)
        table = torch.empty((n, d // 2), dtype=torch.int32, device=cuda_device)
        check(lib.ddt_rope_table(pos.data_ptr(), n, inv_freq.data_ptr(), d, 1.0,
                                 table.data_ptr(), st), "ddt_rope_table")
        outs = []
        for dev_len in (False, True):
            q = torch.zeros((n, hq, d), dtype=torch.bfloat16, device=cuda_device)
            kc = torch.full((hkv, cap, d), 7.0, dtype=torch.bfloat16, device=cuda_device)
            vc = torch.full((hkv, cap, d), 7.0, dtype=torch.bfloat16, device=cuda_device)
            if dev_len:
                past_dev = torch.full((1,), live, dtype=torch.int64, device=cuda_device)
                check(lib.ddt_qk_norm_rope_cache_table_device_past(
                    qkv.data_ptr(), n, hq, hkv, d, qn.data_ptr(), kn.data_ptr(), 1e-6,
                    table.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.stride(0),
                    kc.stride(1), max_past, past_dev.data_ptr(), st), "device past")
            else:
                check(lib.ddt_qk_norm_rope_cache_table(
                    qkv.data_ptr(), n, hq, hkv, d, qn.data_ptr(), kn.data_ptr(), 1e-6,
                    table.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.stride(0),
                    kc.stride(1), live, st), "host past")
            outs.append((q, kc, vc))
        torch.cuda.synchronize()
        for a, b in zip(*outs):
            assert torch.equal(a, b), live
        assert bool((outs[1][1][:, :live] == 7.0).all()) and bool((outs[1][1][:, live + n:] == 7.0).all())
    # out of range: nothing written
    for bad in (max_past + 1, -3):
        q = torch.zeros((n, hq, d), dtype=torch.bfloat16, device=cuda_device)
        kc = torch.full((hkv, cap, d), 7.0, dtype=torch.bfloat16, device=cuda_device)
        vc = torch.full((hkv, cap, d), 7.0, dtype=torch.bfloat16, device=cuda_device)
        past_dev = torch.full((1,), bad, dtype=torch.int64, device=cuda_device)
        check(lib.ddt_qk_norm_rope_cache_table_device_past(
            qkv.data_ptr(), n, hq, hkv, d, qn.data_ptr(), kn.data_ptr(), 1e-6, table.data_ptr(),
            q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1), max_past,
            past_dev.data_ptr(), st), "device past, out of range")
        torch.cuda.synchronize()
        assert bool((q == 0).all()) and bool((kc == 7.0).all()) and bool((vc == 7.0).all())


LOOP_V, LOOP_P, LOOP_BUDGET, LOOP_DEPTHS, LOOP_ROUNDS = 2048, 120, 24, 4, 10


@pytest.fixture(scope="module")
def loop_model(cuda_device):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=LOOP_V, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=128, rope_theta=1e6, max_position_embeddings=4096,
                      rms_norm_eps=1e-6, tie_word_embeddings=False, initializer_range=0.2)
    torch.manual_seed(0)
    return Qwen3ForCausalLM(cfg).to(cuda_device, torch.bfloat16).eval()


def _greedy_continuation(model, tokens, steps, device):
    """The target's own greedy continuation of `tokens` (transformers forward, sdpa)."""
    seq = torch.tensor(tokens, device=device)[None]
    out = []
    with torch.inference_mode():
        for _ in range(steps):
            nxt = int(model(seq).logits[0, -1].argmax())
            out.append(nxt)
            seq = torch.cat([seq, torch.tensor([[nxt]], device=device)], 1)
    return out


def test_one_captured_step_serves_every_round(cuda_device, loop_model):
    """A decode loop (ddtree.py:417-506: verify, walk, compact, start += accepted) whose every
    round replays ONE graph recorded with max_start, against the eager step at the host
    prefix length on a second cache: per round the same tree, the same greedy posterior on
    every decided row (near-ties logged), the same accepted path, next token and commit.
    The stand-in drafter puts the target's greedy continuation on top of random logits, so
    rounds accept several tokens and the prefix crosses a 128-key tile boundary."""
    from mdflash_b200.cache import TreeKVCache
    from mdflash_b200.runner import Qwen3VerifyRunner
    from mdflash_b200.verifier import CapturedStep, TreeVerifier
    from parity_util import posterior_agreement, walk_agrees
    max_start = LOOP_P + LOOP_ROUNDS * (LOOP_DEPTHS + 1)
    cap = max_start + LOOP_BUDGET + 1
    runner = Qwen3VerifyRunner(loop_model)
    caches = [TreeKVCache(2, cap).allocate(2, 128, torch.bfloat16, cuda_device) for _ in range(2)]
    rng = np.random.default_rng(3)
    ids = torch.from_numpy(rng.integers(0, LOOP_V, LOOP_P)).to(cuda_device)
    with torch.inference_mode():
        for c in caches:
            runner.forward(ids, torch.arange(LOOP_P, device=cuda_device), c, 0, None, causal=True)
    torch.cuda.synchronize()
    eager = TreeVerifier(loop_model, caches[0], LOOP_BUDGET, LOOP_DEPTHS, LOOP_V, cuda_device,
                         keep_logits=True, fused=True, runner=runner)
    graphed = TreeVerifier(loop_model, caches[1], LOOP_BUDGET, LOOP_DEPTHS, LOOP_V, cuda_device,
                           fused=True, runner=runner)
    step = CapturedStep(graphed, LOOP_P, max_start=max_start)
    assert caches[1].get_seq_length() == LOOP_P
    tokens = ids.tolist()
    root = torch.tensor([int(rng.integers(0, LOOP_V))], device=cuda_device)
    start = LOOP_P
    compared = 0
    for rnd in range(LOOP_ROUNDS):
        draft = rng.standard_normal((LOOP_DEPTHS, LOOP_V)).astype(np.float32) * 3
        cont = _greedy_continuation(loop_model, tokens + [int(root.item())], LOOP_DEPTHS,
                                    cuda_device)
        draft[np.arange(LOOP_DEPTHS), cont] += 20.0
        logits = torch.from_numpy(draft).to(torch.bfloat16).to(cuda_device)
        ra = eager.step(logits, root, start)
        step.draft_logits.copy_(logits)
        step.root_token.copy_(root)
        rb = step.replay(start)
        torch.cuda.synchronize()
        n = ra.n_nodes
        assert rb.n_nodes == n
        tb = graphed.tree_device_past
        assert torch.equal(eager.tree.parents[:n], tb.parents[:n]), rnd
        assert torch.equal(eager.tree.node_token_ids[:n - 1], tb.node_token_ids[:n - 1]), rnd
        assert torch.equal(eager.tree.verify_pos[:n], tb.verify_pos[:n]), rnd
        ref = ra.logits.float()
        top2 = torch.topk(ref, 2, dim=-1).values
        pa, pb = ra.posterior.cpu().numpy(), rb.posterior.cpu().numpy()
        agree = posterior_agreement(f"loop round {rnd} start {start}", pb, pa,
                                    (top2[:, 0] - top2[:, 1]).cpu().numpy(),
                                    4 * 2.0 ** -7 * ref.abs().max().item())
        assert agree == 1.0, rnd
        ka, kb = int(ra.n_accepted.item()), int(rb.n_accepted.item())
        acc_a = ra.accepted[:ka].tolist()
        if not walk_agrees(acc_a, pb, pa):
            print(f"[loop] round {rnd}: a near-tie on the accepted path; stopping the comparison")
            break
        assert kb == ka and rb.accepted[:kb].tolist() == acc_a, rnd
        assert int(rb.next_token.item()) == int(ra.next_token.item()), rnd
        eager.commit(start, ka)
        graphed.commit(start, kb)
        for la, lb in zip(caches[0].layers, caches[1].layers):
            assert la.length == lb.length == start + ka
            assert _rel_err(lb.keys, la.keys) <= ATTN_TOL
        print(f"[loop] round {rnd}: start {start}, accepted {ka}")
        tokens += eager.tree.verify_ids[ra.accepted[:ka]].tolist()
        start += ka
        root = ra.next_token.clone()
        compared += 1
    assert compared >= 5
    assert start >= LOOP_P + 2 * compared  # several tokens accepted per round on average
    # the recorded step refuses a prefix it was not planned for, on the host
    with pytest.raises(ValueError):
        step.replay(max_start + 1)


def test_device_advanced_rounds_match_host_driven_loop(cuda_device, loop_model):
    """CapturedStep(advance=True): R rounds enqueued back to back, each advancing the device
    start and root itself (ddt_advance_round), with one host sync at the end; against the same
    recorded step driven round by round from the host (replay(start), read, commit) on a
    second cache: the same acceptance lengths, the same committed tokens (the reference's
    output_ids writes, ddtree.py:488-489) and the same final start and cache length."""
    from mdflash_b200.cache import TreeKVCache
    from mdflash_b200.runner import Qwen3VerifyRunner
    from mdflash_b200.verifier import CapturedStep, TreeVerifier
    rounds = 8
    max_start = LOOP_P + 2 * rounds * (LOOP_DEPTHS + 1)
    cap = max_start + LOOP_BUDGET + 1
    runner = Qwen3VerifyRunner(loop_model)
    caches = [TreeKVCache(2, cap).allocate(2, 128, torch.bfloat16, cuda_device) for _ in range(2)]
    rng = np.random.default_rng(5)
    ids = torch.from_numpy(rng.integers(0, LOOP_V, LOOP_P)).to(cuda_device)
    with torch.inference_mode():
        for c in caches:
            runner.forward(ids, torch.arange(LOOP_P, device=cuda_device), c, 0, None, causal=True)
    logits = torch.from_numpy(rng.standard_normal((LOOP_DEPTHS, LOOP_V)).astype(np.float32)
                              * 3).to(torch.bfloat16).to(cuda_device)
    root0 = int(rng.integers(0, LOOP_V))
    steps = []
    for c in caches:
        v = TreeVerifier(loop_model, c, LOOP_BUDGET, LOOP_DEPTHS, LOOP_V, cuda_device, fused=True,
                         runner=runner)
        st = CapturedStep(v, LOOP_P, max_start=max_start, advance=True)
        st.draft_logits.copy_(logits)
        steps.append((v, st))
    # host-driven
    v, st = steps[0]
    st.root_token.fill_(root0)
    start, host_lengths, host_tokens = LOOP_P, [], []
    for _ in range(rounds):
        res = st.replay(start)
        k = int(res.n_accepted.item())
        host_tokens += v.tree_device_past.verify_ids[res.accepted[:k]].tolist()
        v.commit(start, k)
        host_lengths.append(k)
        start += k
        st.root_token.copy_(res.next_token)
    host_tokens.append(int(st.root_token.item()))
    # device-advanced: two batches of rounds, one sync each
    v, st = steps[1]
    st.begin(LOOP_P, root0)
    st.run_rounds(rounds // 2)
    mid, first = st.finish()
    assert caches[1].get_seq_length() == mid
    st.run_rounds(rounds - rounds // 2)
    end, second = st.finish()
    torch.cuda.synchronize()
    print(f"[advance] lengths {first + second}, start {LOOP_P} -> {end}")
    assert first + second == host_lengths
    assert end == start and caches[1].get_seq_length() == end == caches[0].get_seq_length()
    assert st.output_ids[0, LOOP_P:end + 1].tolist() == host_tokens
    for la, lb in zip(caches[0].layers, caches[1].layers):
        assert torch.equal(la.keys, lb.keys) and torch.equal(la.values, lb.values)
    # the host refuses a batch that could pass max_start
    with pytest.raises(ValueError):
        st.run_rounds(2 * rounds)


def test_advance_round_bounds(cuda_device):
    """ddt_advance_round's own writes, and a full output log: dropped writes, status bit 8."""
    dev = cuda_device
    starts = torch.tensor([3, 6], dtype=torch.int64, device=dev)
    rounds = torch.zeros(2, dtype=torch.int32, device=dev)
    n_acc = torch.tensor([2, 3], dtype=torch.int32, device=dev)
    acc = torch.tensor([[0, 2, 0, 0], [0, 1, 3, 0]], dtype=torch.int64, device=dev)
    vids = torch.tensor([[10, 11, 12, 13], [20, 21, 22, 23]], dtype=torch.int64, device=dev)
    nxt = torch.tensor([99, 98], dtype=torch.int64, device=dev)
    roots = torch.zeros(2, dtype=torch.int64, device=dev)
    out = torch.full((2, 9), -7, dtype=torch.int64, device=dev)
    lens = torch.zeros((2, 4), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    K.advance_round(starts, rounds, n_acc, acc, vids, nxt, roots, out, lens, status=status)
    torch.cuda.synchronize()
    assert out[0].tolist() == [-7, -7, -7, 10, 12, 99, -7, -7, -7]
    # request 1: positions 6, 7, 8 fit, 9 (the next token) does not
    assert out[1].tolist() == [-7] * 6 + [20, 21, 23]
    assert starts.tolist() == [5, 9] and rounds.tolist() == [1, 1]
    assert roots.tolist() == [99, 98] and lens[:, 0].tolist() == [2, 3]
    assert int(status.item()) == K.STATUS_LOG_FULL
    with pytest.raises(DDTreeError, match="decode-loop log full"):
        K.check_status(status)
