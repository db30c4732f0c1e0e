"""transformers attention plug-in running the tcgen05 tree-attention kernel.

Registered as ``attn_implementation="ddtree_tree"`` through transformers'
``AttentionInterface`` (transformers/utils/generic.py, modeling_utils.py) with the
signature of ``sdpa_attention_forward`` (transformers/integrations/sdpa_attention.py:40-50),
so an unmodified Qwen3 model runs its verify forward through it:

* tree verify (ddtree.py:467): the ancestor bitmasks come from the active tree context
  (set by this package's ``compile_ddtree_tree`` or ``tree_verify``); when a caller only
  has the reference's additive 4-D mask, the tree block of that mask is converted to
  bitmasks on the device;
* no mask (prefill, plain decode): causal attention, node i sees keys < past + i + 1;
* no mask on a non-causal module (``module.is_causal`` False: the DFlash drafter's attention
  over context + noise block, model/dflash.py:58-102): every query sees every key.

The kernel computes in bf16 with fp32 accumulation; an fp32 model's q / k / v are rounded
to bf16 for it (within the bf16 tolerance of fp32 attention).  Bounded-wait timeouts of the
kernel are reported to a status word (the context's, or the device's default one), which
``follow_verified_tree`` and ``TreeVerifier.check`` read when they sync.
"""
from __future__ import annotations

import threading
from contextlib import contextmanager

import torch

from . import kernels as K

ATTN_IMPLEMENTATION = "ddtree_tree"


class _TreeContext(threading.local):
    def __init__(self):
        self.tree: K.DeviceTree | None = None
        self.past_length: int | None = None
        self.n_nodes: int = 0
        # status word the plug-in's launches report bounded-wait timeouts to (None: the
        # device's default word, kernels.attention_status)
        self.status: torch.Tensor | None = None


_CTX = _TreeContext()


def set_tree_context(tree: "K.DeviceTree | None", past_length: int | None = None,
                     n_nodes: int | None = None) -> None:
    """Makes `tree` the tree the next verify forward attends with (keys [0, past_length)
    are the prefix, [past_length, past_length + n_nodes) the tree)."""
    _CTX.tree = tree
    _CTX.past_length = past_length
    _CTX.n_nodes = (tree.n_nodes if n_nodes is None else n_nodes) if tree is not None else 0


def clear_tree_context() -> None:
    set_tree_context(None)


def get_tree_context():
    return _CTX.tree, _CTX.past_length, _CTX.n_nodes


@contextmanager
def tree_verify(tree: "K.DeviceTree", past_length: int, n_nodes: int | None = None,
                status: torch.Tensor | None = None):
    prev = (_CTX.tree, _CTX.past_length, _CTX.n_nodes, _CTX.status)
    set_tree_context(tree, past_length, n_nodes)
    _CTX.status = status
    try:
        yield
    finally:
        _CTX.tree, _CTX.past_length, _CTX.n_nodes, _CTX.status = prev


def ddtree_attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                             value: torch.Tensor, attention_mask: torch.Tensor | None,
                             dropout: float = 0.0, scaling: float | None = None,
                             is_causal: bool | None = None, **kwargs):
    """query [1, Hq, N, D], key / value [1, Hkv, S, D] -> ([1, N, Hq, D], None)."""
    if dropout not in (0, 0.0):
        raise ValueError("ddtree_tree attention is inference-only (dropout must be 0)")
    if query.shape[0] != 1:
        raise ValueError("ddtree_tree attention supports batch size 1 per request")
    n = query.shape[2]
    s = key.shape[2]
    past = s - n
    tree, ctx_past, ctx_n = get_tree_context()
    st = _CTX.status
    if tree is not None and ctx_n == n and ctx_past == past:
        out = K.tree_attention(query, key, value, tree.anc_bits, past, scale=scaling, status=st)
    elif attention_mask is not None:
        if attention_mask.dim() != 4 or attention_mask.shape[-2] != n or attention_mask.shape[-1] < s:
            raise ValueError("expected the 4-D tree mask [1, 1, N, past + N]")
        bits = K.mask_to_bits(attention_mask[0, 0, :, past:past + n])
        out = K.tree_attention(query, key, value, bits, past, scale=scaling, status=st)
    elif is_causal is False or getattr(module, "is_causal", True) is False:
        # a non-causal module without a mask (the DFlash drafter's context + block
        # attention, model/dflash.py:58-102): every query sees every key
        out = K.tree_attention(query, key, value, None, past, scale=scaling, unmasked=True,
                               status=st)
    else:
        out = K.tree_attention(query, key, value, None, past, scale=scaling, causal=True,
                               status=st)
    return out.unsqueeze(0), None


def register(name: str = ATTN_IMPLEMENTATION) -> str:
    """Registers the plug-in with transformers and returns its implementation name."""
    from transformers import AttentionInterface
    AttentionInterface.register(name, ddtree_attention_forward)
    return name
