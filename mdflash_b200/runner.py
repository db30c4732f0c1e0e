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
                past_dev: torch.Tensor | None = None) -> torch.Tensor:
        """ids, positions: i64 [N] (device).  Writes the N new K/V rows into `cache`
        (a TreeKVCache) at [past_length, past_length + N) and returns logits [N, V] (bf16).
        Tree mode attends with anc_bits; causal=True attends causally (prefill).  Attention
        timeouts go to `status` (default: the device's status word).

        past_dev (i64 [1], device): the prefix length is read from it by the kernels, so that
        a recorded forward serves every prefix length up to past_length (the cache must hold
        past_length + N rows); the cache's host-side length is then left to the caller."""
        h = self._final_hidden(ids, positions, cache, past_length, anc_bits, causal, status,
                               past_dev)
        return torch.matmul(h, self.lm_head.t())

    def forward_posterior(self, ids: torch.Tensor, positions: torch.Tensor, cache,
                          past_length: int, anc_bits: torch.Tensor | None,
                          out: torch.Tensor | None = None,
                          status: torch.Tensor | None = None,
                          past_dev: torch.Tensor | None = None) -> torch.Tensor:
        """The greedy posterior (i64 [N]) of the verify rows without the [N, V] logits: the
        final hidden states go through the fused lm_head -> argmax kernel
        (ddt_lm_head_argmax).  Same cache effects (and past_dev) as forward."""
        h = self._final_hidden(ids, positions, cache, past_length, anc_bits, False, status,
                               past_dev)
        return K.lm_head_argmax(h, self.lm_head, out=out)

    def _final_hidden(self, ids, positions, cache, past_length, anc_bits, causal, status,
                      past_dev=None):
        lib = _lib.load()
        st = self._stream()
        n = ids.numel()
        H, hq, hkv, d = self.hidden, self.q_heads, self.kv_heads, self.head_dim
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
        if past_dev is not None:
            return h
        for layer in cache.layers:
            layer.length = past_length + n
        return h
