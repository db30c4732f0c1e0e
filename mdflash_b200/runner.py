"""Lean Qwen3 verify forward over the weights of a transformers Qwen3ForCausalLM.

transformers' Qwen3 decoder layer (models/qwen3/modeling_qwen3.py:294-330 with
Qwen3Attention :252-291 and Qwen3MLP :70-83) launches about 55 kernels per layer at verify
size, most of them small elementwise ops.  This runner keeps the model's parameters and
its bf16 rounding points but runs each layer as

    ddt_add_rmsnorm          residual add + input_layernorm
    GEMM                     q/k/v projections (one cuBLAS GEMM on the concatenated weight)
    ddt_qk_norm_rope_cache_table
                             q_norm / k_norm, rotary embedding, K/V written into the cache
    ddt_tree_attn            tree attention (tcgen05)
    GEMM                     o_proj
    ddt_add_rmsnorm          residual add + post_attention_layernorm
    GEMM                     gate/up projections (one GEMM on the concatenated weight)
    ddt_silu_mul             SiLU(gate) * up
    GEMM                     down_proj

followed by the final norm and lm_head.  The rotary cos / sin of the forward's positions are
built once (ddt_rope_table) and read by every layer.  It is used by TreeVerifier(fused=True).
"""
from __future__ import annotations

import torch

from . import _lib
from . import kernels as K
from ._lib import check


def gemm_chunk(rows: int, max_chunk: int = 2048, align: int = 128) -> int:
    """Rows per projection GEMM of a batched verify forward over `rows` tree rows: the fewest
    chunks of at most `max_chunk` rows, each a multiple of `align` (the rows are padded up to
    a whole number of chunks)."""
    if rows <= 0 or max_chunk <= 0 or align <= 0 or max_chunk % align:
        raise ValueError("rows, max_chunk and align must be positive, max_chunk a multiple of align")
    pieces = -(-rows // max_chunk)
    return -(-(-(-rows // pieces)) // align) * align


class Qwen3VerifyRunner:
    def __init__(self, model):
        cfg = model.config
        self.cfg = cfg
        self.hidden = cfg.hidden_size
        self.q_heads = cfg.num_attention_heads
        self.kv_heads = cfg.num_key_value_heads
        self.head_dim = getattr(cfg, "head_dim", self.hidden // self.q_heads)
        self.inter = cfg.intermediate_size
        self.eps = float(cfg.rms_norm_eps)
        inner = model.model
        self.embed = inner.embed_tokens.weight
        self.final_norm = inner.norm.weight
        self.lm_head = model.lm_head.weight
        rot = inner.rotary_emb
        self.inv_freq = rot.inv_freq.to(torch.float32).contiguous()
        self.rope_scale = float(getattr(rot, "attention_scaling", 1.0))
        self.scaling = self.head_dim ** -0.5
        self.layers = []
        with torch.no_grad():
            for layer in inner.layers:
                a, m = layer.self_attn, layer.mlp
                for lin in (a.q_proj, a.k_proj, a.v_proj, a.o_proj):
                    if lin.bias is not None:
                        raise ValueError("attention projections with bias are not supported")
                self.layers.append(dict(
                    w_qkv=torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0),
                    w_o=a.o_proj.weight,
                    w_gu=torch.cat([m.gate_proj.weight, m.up_proj.weight], 0),
                    w_down=m.down_proj.weight,
                    ln1=layer.input_layernorm.weight, ln2=layer.post_attention_layernorm.weight,
                    qn=a.q_norm.weight, kn=a.k_norm.weight))
        self.device = self.embed.device

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def forward(self, ids: torch.Tensor, positions: torch.Tensor, cache, past_length: int,
                anc_bits: torch.Tensor | None, causal: bool = False,
                status: torch.Tensor | None = None,
                past_dev: torch.Tensor | None = None,
                features: torch.Tensor | None = None,
                feature_layers: list[int] | None = None) -> torch.Tensor:
        """ids, positions: i64 [N] (device).  Writes the N new K/V rows into `cache`
        (a TreeKVCache) at [past_length, past_length + N) and returns logits [N, V] (bf16).
        Tree mode attends with anc_bits; causal=True attends causally (prefill).  Attention
        timeouts go to `status` (default: the device's status word).

        past_dev (i64 [1], device): the prefix length is read from it by the kernels, so that
        a recorded forward serves every prefix length up to past_length (the cache must hold
        past_length + N rows); the cache's host-side length is then left to the caller.

        features [N, len(feature_layers) * hidden] (bf16): receives the target's context
        features of the drafter, extract_context_feature(output.hidden_states, layer_ids)
        (model/utils.py:17-26): for layer id i, hidden_states[i + 1] in transformers' sense,
        i.e. the residual stream after decoder layer i, or the final normed state for the
        last layer."""
        h = self._final_hidden(ids, positions, cache, past_length, anc_bits, causal, status,
                               past_dev, features, feature_layers)
        return torch.matmul(h, self.lm_head.t())

    def forward_posterior(self, ids: torch.Tensor, positions: torch.Tensor, cache,
                          past_length: int, anc_bits: torch.Tensor | None,
                          out: torch.Tensor | None = None,
                          status: torch.Tensor | None = None,
                          past_dev: torch.Tensor | None = None,
                          features: torch.Tensor | None = None,
                          feature_layers: list[int] | None = None) -> torch.Tensor:
        """The greedy posterior (i64 [N]) of the verify rows without the [N, V] logits: the
        final hidden states go through the fused lm_head -> argmax kernel
        (ddt_lm_head_argmax).  Same cache effects (and past_dev, features) as forward."""
        h = self._final_hidden(ids, positions, cache, past_length, anc_bits, False, status,
                               past_dev, features, feature_layers)
        return K.lm_head_argmax(h, self.lm_head, out=out)

    def forward_batch(self, ids: torch.Tensor, positions: torch.Tensor,
                      segments: list[tuple[int, int]], caches: list, pasts: list[int],
                      anc_bits: list[torch.Tensor], status: torch.Tensor | None = None,
                      chunk: int = 2048, lanes: int = 1, kv_splits: int = 0) -> torch.Tensor:
        """The verify forward of many requests at once.  ids / positions: i64 [T_pad] (device;
        request r's tree rows at segments[r] = (offset, rows); the rows after the last segment
        are padding, T_pad a multiple of `chunk`).  Request r's K/V rows go into caches[r] at
        pasts[r], and its rows attend to that cache under anc_bits[r].  The norms and the
        projections run over all rows, the projections in GEMMs of exactly `chunk` rows, so
        that a row's result does not depend on which other requests share the batch; the
        K/V writes and the attention run per request, spread over `lanes` streams (kv_splits:
        the attention's key splits per request, 0 lets the library choose; 1 runs one CTA per
        work unit and no merge, leaving the GPU to the other lanes' launches).  Returns
        logits [T_pad, V] (bf16; padding rows are finite and meaningless)."""
        lib = _lib.load()
        T = ids.numel()
        if T % chunk:
            raise ValueError(f"{T} rows is not a multiple of the chunk ({chunk})")
        if not (len(segments) == len(caches) == len(pasts) == len(anc_bits)):
            raise ValueError("one segment, cache, prefix length and tree per request")
        for (off, n), c, p in zip(segments, caches, pasts):
            if off < 0 or n <= 0 or off + n > T or p < 0 or p + n > c.capacity:
                raise ValueError(f"segment ({off}, {n}) at prefix {p} does not fit")
        st = self._stream()
        dev = ids.device
        H, hq, hkv, d = self.hidden, self.q_heads, self.kv_heads, self.head_dim
        x = torch.nn.functional.embedding(ids.view(-1), self.embed)  # [T, H] bf16
        h = torch.empty_like(x)
        q = torch.zeros((T, hq, d), dtype=x.dtype, device=dev)
        attn = torch.zeros((T, hq, d), dtype=x.dtype, device=dev)  # padding rows stay 0
        qkv = torch.empty((T, (hq + 2 * hkv) * d), dtype=x.dtype, device=dev)
        o = torch.empty((T, H), dtype=x.dtype, device=dev)
        gu = torch.empty((T, 2 * self.inter), dtype=x.dtype, device=dev)
        act = torch.empty((T, self.inter), dtype=x.dtype, device=dev)
        delta = torch.empty((T, H), dtype=x.dtype, device=dev)
        rope = torch.empty((T, d // 2), dtype=torch.int32, device=dev)
        check(lib.ddt_rope_table(positions.data_ptr(), T, self.inv_freq.data_ptr(), d,
                                 self.rope_scale, rope.data_ptr(), st), "ddt_rope_table")
        K.STATS.launches += 1

        def gemm(a, w, out):
            for c0 in range(0, T, chunk):
                torch.matmul(a[c0:c0 + chunk], w.t(), out=out[c0:c0 + chunk])
            K.STATS.launches += T // chunk

        main = torch.cuda.current_stream(dev)
        side = [torch.cuda.Stream(dev) for _ in range(lanes)] if lanes > 1 else None
        first = True
        for li, w in enumerate(self.layers):
            check(lib.ddt_add_rmsnorm(x.data_ptr(), None if first else delta.data_ptr(),
                                      w["ln1"].data_ptr(), T, H, self.eps, x.data_ptr(),
                                      h.data_ptr(), st), "ddt_add_rmsnorm")
            first = False
            gemm(h, w["w_qkv"], qkv)
            if side:
                for sst in side:
                    sst.wait_stream(main)
            for r, ((off, n), cache, past) in enumerate(zip(segments, caches, pasts)):
                ln = r % lanes
                sst = side[ln] if side else main
                with torch.cuda.stream(sst), K.WORKSPACES.lane(ln):
                    layer = cache.layers[li]
                    kbuf, vbuf = layer.k_buf[0], layer.v_buf[0]
                    check(lib.ddt_qk_norm_rope_cache_table(
                        qkv[off].data_ptr(), n, hq, hkv, d, w["qn"].data_ptr(),
                        w["kn"].data_ptr(), self.eps, rope[off].data_ptr(), q[off].data_ptr(),
                        kbuf.data_ptr(), vbuf.data_ptr(), kbuf.stride(0), kbuf.stride(1), past,
                        sst.cuda_stream), "ddt_qk_norm_rope_cache_table")
                    s_len = past + n
                    K.tree_attention(q[off:off + n], kbuf[:, :s_len], vbuf[:, :s_len],
                                     anc_bits[r], past, scale=self.scaling, status=status,
                                     out=attn[off:off + n], kv_splits=kv_splits)
                K.STATS.launches += 1
            if side:
                for sst in side:
                    main.wait_stream(sst)
            gemm(attn.view(T, hq * d), w["w_o"], o)
            check(lib.ddt_add_rmsnorm(x.data_ptr(), o.data_ptr(), w["ln2"].data_ptr(), T, H,
                                      self.eps, x.data_ptr(), h.data_ptr(), st), "ddt_add_rmsnorm")
            gemm(h, w["w_gu"], gu)
            check(lib.ddt_silu_mul(gu.data_ptr(), T, self.inter, act.data_ptr(), st),
                  "ddt_silu_mul")
            gemm(act, w["w_down"], delta)
            K.STATS.launches += 3
        check(lib.ddt_add_rmsnorm(x.data_ptr(), delta.data_ptr(), self.final_norm.data_ptr(), T,
                                  H, self.eps, x.data_ptr(), h.data_ptr(), st), "ddt_add_rmsnorm")
        K.STATS.launches += 1
        logits = torch.empty((T, self.lm_head.shape[0]), dtype=x.dtype, device=dev)
        gemm(h, self.lm_head, logits)
        return logits

    def _feature_slots(self, features, feature_layers, n):
        """hidden-state index (transformers' hidden_states[i], i = layer id + 1) -> the
        column slices of `features` it fills."""
        if features is None:
            return {}
        L = len(self.layers)
        H = self.hidden
        if not feature_layers or features.shape != (n, len(feature_layers) * H) or \
                features.dtype != torch.bfloat16:
            raise ValueError("features must be bf16 [N, len(feature_layers) * hidden]")
        slots = {}
        for j, lid in enumerate(feature_layers):
            if not -1 <= lid < L:
                raise ValueError(f"feature layer {lid} outside [-1, {L})")
            slots.setdefault(lid + 1, []).append(features[:, j * H:(j + 1) * H])
        return slots

    def _final_hidden(self, ids, positions, cache, past_length, anc_bits, causal, status,
                      past_dev=None, features=None, feature_layers=None):
        lib = _lib.load()
        st = self._stream()
        n = ids.numel()
        H, hq, hkv, d = self.hidden, self.q_heads, self.kv_heads, self.head_dim
        slots = self._feature_slots(features, feature_layers, n)
        x = torch.nn.functional.embedding(ids.view(-1), self.embed)  # [N, H] bf16
        h = torch.empty_like(x)
        q = torch.empty((n, hq, d), dtype=x.dtype, device=x.device)
        act = torch.empty((n, self.inter), dtype=x.dtype, device=x.device)
        rope = torch.empty((n, d // 2), dtype=torch.int32, device=x.device)
        check(lib.ddt_rope_table(positions.data_ptr(), n, self.inv_freq.data_ptr(), d,
                                 self.rope_scale, rope.data_ptr(), st), "ddt_rope_table")
        K.STATS.launches += 1
        delta = None
        for li, w in enumerate(self.layers):
            layer = cache.layers[li]
            kbuf, vbuf = layer.k_buf[0], layer.v_buf[0]  # [Hkv, cap, D]
            check(lib.ddt_add_rmsnorm(x.data_ptr(), delta.data_ptr() if delta is not None else None,
                                      w["ln1"].data_ptr(), n, H, self.eps, x.data_ptr(),
                                      h.data_ptr(), st), "ddt_add_rmsnorm")
            for dst in slots.get(li, ()):  # the residual stream entering layer li
                dst.copy_(x)
            qkv = torch.matmul(h, w["w_qkv"].t())
            if past_dev is None:
                check(lib.ddt_qk_norm_rope_cache_table(
                    qkv.data_ptr(), n, hq, hkv, d, w["qn"].data_ptr(), w["kn"].data_ptr(),
                    self.eps, rope.data_ptr(), q.data_ptr(), kbuf.data_ptr(), vbuf.data_ptr(),
                    kbuf.stride(0), kbuf.stride(1), past_length, st),
                    "ddt_qk_norm_rope_cache_table")
            else:
                check(lib.ddt_qk_norm_rope_cache_table_device_past(
                    qkv.data_ptr(), n, hq, hkv, d, w["qn"].data_ptr(), w["kn"].data_ptr(),
                    self.eps, rope.data_ptr(), q.data_ptr(), kbuf.data_ptr(), vbuf.data_ptr(),
                    kbuf.stride(0), kbuf.stride(1), past_length, past_dev.data_ptr(), st),
                    "ddt_qk_norm_rope_cache_table_device_past")
            K.STATS.launches += 3
            s = past_length + n
            attn = K.tree_attention(q, kbuf[:, :s], vbuf[:, :s], anc_bits, past_length,
                                    scale=self.scaling, causal=causal, status=status,
                                    past_dev=past_dev)
            o = torch.matmul(attn.view(n, hq * d), w["w_o"].t())
            check(lib.ddt_add_rmsnorm(x.data_ptr(), o.data_ptr(), w["ln2"].data_ptr(), n, H,
                                      self.eps, x.data_ptr(), h.data_ptr(), st), "ddt_add_rmsnorm")
            gu = torch.matmul(h, w["w_gu"].t())
            check(lib.ddt_silu_mul(gu.data_ptr(), n, self.inter, act.data_ptr(), st),
                  "ddt_silu_mul")
            delta = torch.matmul(act, w["w_down"].t())
            K.STATS.launches += 2
        check(lib.ddt_add_rmsnorm(x.data_ptr(), delta.data_ptr(), self.final_norm.data_ptr(), n, H,
                                  self.eps, x.data_ptr(), h.data_ptr(), st), "ddt_add_rmsnorm")
        K.STATS.launches += 1
        for dst in slots.get(len(self.layers), ()):  # the last entry: the final normed state
            dst.copy_(h)
        if past_dev is not None:
            return h
        for layer in cache.layers:
            layer.length = past_length + n
        return h
