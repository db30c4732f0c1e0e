"""GPU parity of the fused lm_head -> greedy posterior (ddt_lm_head_argmax).

* Bit-exact with ddt_argmax on the same logits: the kernel can also write the bf16 logits it
  took the argmax over, and the argmax kernel on them must give the same posterior, ties
  included.
* Those logits are the bf16 rounding of fp32 dot products: element-wise within one bf16 step
  (2^-8 relative, with the row RMS as the floor) of an fp32 reference GEMM.
* Against the unfused path (torch.matmul in bf16, then argmax), the posteriors agree on >=
  99.9% of the rows whose top-1 / top-2 gap exceeds 4 bf16 steps of the largest logit;
  near-ties are logged.
"""
import numpy as np
import pytest
import torch

from mdflash_b200 import kernels as K
from parity_util import posterior_agreement

pytestmark = pytest.mark.gpu


def _inputs(device, n, H, V, seed, scale=1.0):
    g = torch.Generator(device=device).manual_seed(seed)
    h = (torch.randn((n, H), generator=g, device=device) * scale).to(torch.bfloat16)
    w = (torch.randn((V, H), generator=g, device=device) * (H ** -0.5)).to(torch.bfloat16)
    return h, w


def _check(h, w, label):
    n, V = h.shape[0], w.shape[0]
    logits = torch.empty((n, V), dtype=torch.bfloat16, device=h.device)
    post = K.lm_head_argmax(h, w, logits_out=logits)
    again = K.lm_head_argmax(h, w)  # without the logits output; the workspace was cleared
    torch.cuda.synchronize()
    K.check_status(K.attention_status(h.device), "ddt_lm_head_argmax")
    assert torch.equal(post, again)
    # (1) bit-exact with the argmax kernel on the same logits
    assert torch.equal(post, K.argmax(logits))
    # (2) the logits are bf16(fp32 dot products)
    ref32 = h.float() @ w.float().t()
    err = (logits.float() - ref32).abs()
    floor = torch.maximum(ref32.abs(), ref32.pow(2).mean(-1, keepdim=True).sqrt())
    assert (err / floor).max().item() <= 2.0 ** -8 + 1e-6, label
    # (3) against the unfused bf16 GEMM + argmax
    unfused = torch.matmul(h, w.t())
    top2 = torch.topk(unfused.float(), 2, dim=-1).values
    tie_gap = 4 * 2.0 ** -7 * unfused.float().abs().max().item()
    frac = posterior_agreement(label, post.cpu().numpy(), unfused.float().argmax(-1).cpu().numpy(),
                               (top2[:, 0] - top2[:, 1]).cpu().numpy(), tie_gap)
    assert frac >= 0.999
    return post


@pytest.mark.parametrize("n,H,V,seed", [
    (257, 4096, 151936, 0),   # Qwen3-8B verify shape (256-node tree + root)
    (33, 1024, 151936, 1),    # Qwen3-0.6B shape, 32-node tree
    (1, 256, 1000, 2),        # one row, vocabulary not a multiple of 128
    (144, 512, 4096, 3),      # exactly the first part of a group
    (145, 512, 4096, 4),      # one row into the second part
    (600, 1024, 5000, 5),     # three groups of verify rows (272 + 272 + 56)
])
def test_lm_head_argmax_shapes(cuda_device, n, H, V, seed):
    h, w = _inputs(cuda_device, n, H, V, seed)
    _check(h, w, f"lm_head n={n} H={H} V={V}")


def test_lm_head_argmax_ties_and_nan(cuda_device):
    """Equal best logits go to the lowest index, also across vocabulary tiles and CTAs; a
    NaN logit wins like in torch.argmax."""
    n, H, V = 40, 256, 3000
    h, w = _inputs(cuda_device, n, H, V, 7)
    big = torch.ones((1, H), device=cuda_device, dtype=torch.bfloat16) * 0.5
    h = h.abs()  # positive hidden states: the all-0.5 row wins every dot product
    for v in (2999, 1700, 130, 131):
        w[v] = big[0]
    post = K.lm_head_argmax(h, w)
    torch.cuda.synchronize()
    assert post.tolist() == [130] * n
    w[2500, 3] = float("nan")
    post = K.lm_head_argmax(h, w)
    torch.cuda.synchronize()
    assert post.tolist() == [2500] * n


def test_lm_head_argmax_strided_hidden(cuda_device):
    """Hidden states as a row view of a wider buffer (the runner's layout)."""
    n, H, V = 65, 512, 7000
    h, w = _inputs(cuda_device, n, H, V, 9)
    wide = torch.zeros((n, H + 64), dtype=torch.bfloat16, device=cuda_device)
    wide[:, :H] = h
    a = K.lm_head_argmax(wide[:, :H], w)
    b = K.lm_head_argmax(h, w)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
