"""The DDTree decode loop on this package's verify path.

``ddtree_generate`` keeps the signature and the results of the reference's loop
(ddtree.py:338-530): prefill, then rounds of draft -> tree build -> compile -> tree-masked
verify -> greedy posterior -> accept walk -> KV compaction, until ``max_new_tokens`` are
committed or a stop token appears.  Every step of a round runs through this package: the tree
build, compile, walk and compaction of :mod:`mdflash_b200.ddtree`, the ``ddtree_tree``
attention plug-in for the target's verify (and prefill) attention, and ``ddt_argmax`` for the
greedy posterior.  The drafter is any module with the DFlash draft model's call signature
(``model(target_hidden=..., noise_embedding=..., position_ids=..., past_key_values=...,
use_cache=..., is_causal=False)`` returning hidden states, and ``model.target_layer_ids``).
"""
from __future__ import annotations

import time
from types import SimpleNamespace

import torch
from transformers import DynamicCache

from . import attention as A
from . import ddtree as D
from . import kernels as K


def _context_feature(hidden_states, layer_ids):
    """model/utils.py:17-26: the hidden states after the drafter's target layers, concatenated."""
    return torch.cat([hidden_states[i + 1] for i in layer_ids], dim=-1)


def _greedy(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    """model/utils.py:28-35 sample(): argmax at temperature < 1e-5 (ddt_argmax), else a draw
    from softmax(logits / T)."""
    if temperature < 1e-5:
        return K.argmax(logits)
    b, n, v = logits.shape
    probs = torch.softmax(logits.view(-1, v).float() / temperature, dim=-1)
    return torch.multinomial(probs, num_samples=1).view(b, n)


@torch.inference_mode()
def ddtree_generate(model, target, input_ids: torch.Tensor, mask_token_id: int,
                    max_new_tokens: int, block_size: int, stop_token_ids, temperature: float = 0.0,
                    tree_budget: int | None = None) -> SimpleNamespace:
    """ddtree.py:338-530 on the B200 path (block_size > 1).  Returns output_ids (CPU),
    num_input_tokens, num_output_tokens, acceptance_lengths, decode_rounds and timings."""
    if block_size <= 1:
        raise ValueError("block_size must be > 1 (the tree path)")
    dev = input_ids.device
    A.register()
    target.config._attn_implementation = A.ATTN_IMPLEMENTATION
    n_in = input_ids.shape[1]
    max_length = n_in + max_new_tokens
    horizon = block_size - 1
    budget = horizon if tree_budget is None else max(tree_budget, 0)
    max_nodes = 1 + budget
    out_ids = torch.full((1, max_length + max_nodes), mask_token_id, dtype=torch.long, device=dev)
    positions = torch.arange(out_ids.shape[1], device=dev).unsqueeze(0)
    stop = None if stop_token_ids is None else torch.tensor(stop_token_ids, device=dev)
    ids_buf = torch.empty((1, max_nodes), dtype=torch.long, device=dev)
    pos_buf = torch.empty((1, max_nodes), dtype=torch.long, device=dev)
    mask_buf = torch.zeros((1, 1, max_nodes, max_length + max_nodes), dtype=target.dtype, device=dev)
    vis_buf = torch.empty((max_nodes, max_nodes), dtype=torch.bool, device=dev)
    cache_target, cache_draft = DynamicCache(), DynamicCache()

    t0 = time.perf_counter()
    out = target(input_ids, position_ids=positions[:, :n_in], past_key_values=cache_target,
                 use_cache=True, logits_to_keep=1, output_hidden_states=True)
    out_ids[:, :n_in] = input_ids
    out_ids[:, n_in:n_in + 1] = _greedy(out.logits, temperature)
    target_hidden = _context_feature(out.hidden_states, model.target_layer_ids)
    ttft = time.perf_counter() - t0

    start = n_in
    acceptance = []
    prev_start = prev_len = 0
    t1 = time.perf_counter()
    while start < max_length:
        block = out_ids[:, start:start + block_size].clone()
        root = block[:, :1]
        noise = target.model.embed_tokens(block)
        draft_hidden = model(target_hidden=target_hidden, noise_embedding=noise,
                             position_ids=positions[:, cache_draft.get_seq_length():start + block_size],
                             past_key_values=cache_draft, use_cache=True, is_causal=False)
        draft_logits = target.lm_head(draft_hidden[:, -horizon:, :])
        cache_draft.crop(start)
        node_ids, depths, parents, child_maps, vis, _ = D.build_ddtree_tree(draft_logits[0], budget)
        v_ids, v_pos, v_mask, prev_start, prev_len = D.compile_ddtree_tree(
            root[0, 0], start, node_ids, depths, vis, start, target.dtype, dev, ids_buf, pos_buf,
            mask_buf, vis_buf, prev_start, prev_len)
        out = target(v_ids, position_ids=v_pos, attention_mask=v_mask,
                     past_key_values=cache_target, use_cache=True, output_hidden_states=True)
        posterior = _greedy(out.logits, temperature)
        accepted, next_token = D.follow_verified_tree(child_maps, posterior)
        acc_t = torch.tensor(accepted, dtype=torch.long, device=dev)
        out_ids[:, start:start + len(accepted)] = v_ids.index_select(1, acc_t)
        out_ids[:, start + len(accepted)] = next_token
        D.compact_dynamic_cache(cache_target, start, accepted)
        target_hidden = _context_feature(out.hidden_states, model.target_layer_ids).index_select(1, acc_t)
        acceptance.append(len(accepted))
        start += len(accepted)
        if stop is not None and torch.isin(out_ids[0, start - len(accepted):start + 1], stop).any():
            break
    A.clear_tree_context()
    out_ids = out_ids[:, :max_length]
    out_ids = out_ids[:, out_ids[0] != mask_token_id]
    if stop is not None:
        hits = torch.isin(out_ids[0][n_in:], stop).nonzero(as_tuple=True)[0]
        if hits.numel() > 0:
            out_ids = out_ids[:, :n_in + hits[0] + 1]
    n_out = out_ids.shape[1] - n_in
    decode = time.perf_counter() - t1
    return SimpleNamespace(output_ids=out_ids.cpu(), num_input_tokens=n_in,
                           num_output_tokens=n_out, time_to_first_token=ttft,
                           time_per_output_token=decode / max(n_out, 1),
                           acceptance_lengths=acceptance, decode_rounds=len(acceptance))
