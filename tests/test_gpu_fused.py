"""GPU parity of the fused elementwise stages of the verify forward (csrc/qwen3_fused.cu)
against the transformers Qwen3 code they replace.

* ddt_add_rmsnorm vs the residual add + Qwen3RMSNorm (modeling_qwen3.py:59-64): the residual
  is bit-exact (one bf16 add); the normed output within two bf16 steps of transformers' (the
  mean of squares is summed in another order, which can move a rounding), with >= 99% of
  the elements identical.
* ddt_rope_table + ddt_qk_norm_rope_cache_table vs ddt_qk_norm_rope_cache: bit-identical (the
  table holds the values the inline path computes), and both vs q_norm / k_norm +
  Qwen3RotaryEmbedding + apply_rotary_pos_emb (:137-181, :263-264) within two bf16 steps of
  the head's RMS, with >= 99% identical and the V rows copied bit-exactly into the cache.
* ddt_silu_mul vs act_fn(gate) * up (:81-83): bit-exact.
"""
import pytest
import torch

from mdflash_b200 import _lib
from mdflash_b200._lib import check
from parity_util import elem_rel_err

pytestmark = pytest.mark.gpu
STEP = 2.0 ** -8  # one bf16 step, relative


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _within_steps(ours, ref, label, min_exact=0.99):
    """Element-wise within two bf16 steps, relative with the row RMS as the floor."""
    o, r = ours.float(), ref.float()
    err = elem_rel_err(o, r)
    exact = (o == r).float().mean().item()
    print(f"[{label}] max rel err {err:.3e}, identical {exact:.5f}")
    assert err <= 2 * STEP * 1.0001, label
    assert exact >= min_exact, label


@pytest.mark.parametrize("rows,hidden,with_delta", [
    (257, 4096, True), (257, 4096, False), (33, 1024, True), (65, 2560, True), (17, 5120, True),
    (9, 8192, True), (3, 16384, True), (1, 8, True)])
def test_add_rmsnorm_matches_transformers(cuda_device, rows, hidden, with_delta):
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
    g = torch.Generator(device=cuda_device).manual_seed(hidden + rows)
    x = (torch.randn((rows, hidden), generator=g, device=cuda_device) * 2).to(torch.bfloat16)
    d = (torch.randn((rows, hidden), generator=g, device=cuda_device)).to(torch.bfloat16)
    norm = Qwen3RMSNorm(hidden, eps=1e-6).to(cuda_device, torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn((hidden,), generator=g, device=cuda_device))
    res_ref = x + d if with_delta else x.clone()
    with torch.no_grad():
        out_ref = norm(res_ref)
    res = torch.empty_like(x)
    out = torch.empty_like(x)
    lib = _lib.load()
    check(lib.ddt_add_rmsnorm(x.data_ptr(), d.data_ptr() if with_delta else None,
                              norm.weight.data_ptr(), rows, hidden, 1e-6, res.data_ptr(),
                              out.data_ptr(), _stream(cuda_device)), "ddt_add_rmsnorm")
    # in place (residual_out aliases x), as the runner calls it
    xi = x.clone()
    out2 = torch.empty_like(x)
    check(lib.ddt_add_rmsnorm(xi.data_ptr(), d.data_ptr() if with_delta else None,
                              norm.weight.data_ptr(), rows, hidden, 1e-6, xi.data_ptr(),
                              out2.data_ptr(), _stream(cuda_device)), "ddt_add_rmsnorm")
    torch.cuda.synchronize()
    assert torch.equal(res, res_ref) and torch.equal(xi, res_ref)
    assert torch.equal(out, out2)
    _within_steps(out, out_ref, f"add_rmsnorm {rows}x{hidden}")


@pytest.mark.parametrize("rows,inter", [(257, 12288), (33, 3072), (1, 8), (3, 24), (7, 9728)])
def test_silu_mul_matches_transformers(cuda_device, rows, inter):
    g = torch.Generator(device=cuda_device).manual_seed(rows * 7 + inter)
    gu = (torch.randn((rows, 2 * inter), generator=g, device=cuda_device) * 3).to(torch.bfloat16)
    gu[0, :8] = torch.tensor([0.0, -0.0, 88.0, -88.0, 1e-30, -1e-30, 20.0, -20.0])
    out = torch.empty((rows, inter), dtype=torch.bfloat16, device=cuda_device)
    check(_lib.load().ddt_silu_mul(gu.data_ptr(), rows, inter, out.data_ptr(),
                                   _stream(cuda_device)), "ddt_silu_mul")
    ref = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def _rope_case(dev, n, hq, hkv, past, seed, cap=None):
    g = torch.Generator(device=dev).manual_seed(seed)
    D = 128
    qkv = (torch.randn((n, (hq + 2 * hkv) * D), generator=g, device=dev) * 2).to(torch.bfloat16)
    qw = (1 + 0.2 * torch.randn((D,), generator=g, device=dev)).to(torch.bfloat16)
    kw = (1 + 0.2 * torch.randn((D,), generator=g, device=dev)).to(torch.bfloat16)
    pos = past + torch.randperm(n, generator=g, device=dev)  # tree positions are not sorted
    cap = cap or past + n + 8
    return qkv, qw, kw, pos.to(torch.int64), cap


def _run_rope(dev, qkv, qw, kw, pos, n, hq, hkv, past, cap, inv_freq, scale, table):
    D = 128
    lib = _lib.load()
    q = torch.empty((n, hq, D), dtype=torch.bfloat16, device=dev)
    kc = torch.zeros((hkv, cap, D), dtype=torch.bfloat16, device=dev)
    vc = torch.zeros((hkv, cap, D), dtype=torch.bfloat16, device=dev)
    st = _stream(dev)
    if table:
        tab = torch.empty((n, D // 2), dtype=torch.int32, device=dev)
        check(lib.ddt_rope_table(pos.data_ptr(), n, inv_freq.data_ptr(), D, scale,
                                 tab.data_ptr(), st), "ddt_rope_table")
        check(lib.ddt_qk_norm_rope_cache_table(qkv.data_ptr(), n, hq, hkv, D, qw.data_ptr(),
                                               kw.data_ptr(), 1e-6, tab.data_ptr(), q.data_ptr(),
                                               kc.data_ptr(), vc.data_ptr(), kc.stride(0),
                                               kc.stride(1), past, st),
              "ddt_qk_norm_rope_cache_table")
    else:
        check(lib.ddt_qk_norm_rope_cache(qkv.data_ptr(), n, hq, hkv, D, qw.data_ptr(),
                                         kw.data_ptr(), 1e-6, pos.data_ptr(), inv_freq.data_ptr(),
                                         scale, q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                         kc.stride(0), kc.stride(1), past, st),
              "ddt_qk_norm_rope_cache")
    return q, kc, vc


@pytest.mark.parametrize("n,hq,hkv,past,theta,scale", [
    (257, 32, 8, 8192, 1e6, 1.0), (33, 16, 8, 4096, 1e6, 1.0), (513, 32, 8, 131072, 1e6, 1.0),
    (5, 4, 2, 0, 1e4, 1.0), (64, 8, 4, 40000, 1e6, 0.75)])
def test_qk_norm_rope_cache_matches_transformers(cuda_device, n, hq, hkv, past, theta, scale):
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import (Qwen3RMSNorm, Qwen3RotaryEmbedding,
                                                          apply_rotary_pos_emb)
    dev, D = cuda_device, 128
    qkv, qw, kw, pos, cap = _rope_case(dev, n, hq, hkv, past, n + hq + past)
    cfg = Qwen3Config(hidden_size=hq * D, num_attention_heads=hq, num_key_value_heads=hkv,
                      head_dim=D, rope_theta=theta, max_position_embeddings=262144)
    rot = Qwen3RotaryEmbedding(cfg).to(dev)
    rot.attention_scaling = scale
    inv_freq = rot.inv_freq.to(torch.float32).contiguous()
    q_t, k_t, v_t = _run_rope(dev, qkv, qw, kw, pos, n, hq, hkv, past, cap, inv_freq, scale, True)
    q_i, k_i, v_i = _run_rope(dev, qkv, qw, kw, pos, n, hq, hkv, past, cap, inv_freq, scale, False)
    torch.cuda.synchronize()
    # the table path is the inline path
    assert torch.equal(q_t, q_i) and torch.equal(k_t, k_i) and torch.equal(v_t, v_i)
    # transformers: q_norm / k_norm over head_dim, then the rotary embedding
    qn, kn = Qwen3RMSNorm(D, eps=1e-6).to(dev, torch.bfloat16), Qwen3RMSNorm(D, eps=1e-6).to(
        dev, torch.bfloat16)
    with torch.no_grad():
        qn.weight.copy_(qw)
        kn.weight.copy_(kw)
        x = qkv.view(n, hq + 2 * hkv, D)
        q_ref = qn(x[:, :hq]).transpose(0, 1)[None]            # [1, hq, n, D]
        k_ref = kn(x[:, hq:hq + hkv]).transpose(0, 1)[None]    # [1, hkv, n, D]
        cos, sin = rot(qkv[None], pos[None])
        q_ref, k_ref = apply_rotary_pos_emb(q_ref, k_ref, cos, sin)
    _within_steps(q_t, q_ref[0].transpose(0, 1), f"q n={n} P={past}")
    _within_steps(k_t[:, past:past + n], k_ref[0], f"k n={n} P={past}")
    assert torch.equal(v_t[:, past:past + n], x[:, hq + hkv:].transpose(0, 1))
    # rows outside [past, past + n) are untouched
    assert not k_t[:, :past].any() and not k_t[:, past + n:].any()
