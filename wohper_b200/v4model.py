"""A DeepSeek-V4 decode step composed from the library's kernels.

The host mirror of the reference's per-token model pass
(run_model_for_one_token, src/server/generation.rs:1822) for the layers'
compute: each layer is phase 1 (compute_layer_deepseek_mhc_phase1,
src/compute.rs:1498-1641) and phase 2 (compute_layer_deepseek_mhc_phase2,
src/compute.rs:1644-1700):

    residual = x;  y, post, comb = hc_pre(hc_attn, x)        (wh_hc_pre)
    y = rms_norm(y, input_layernorm)                          (wh_rms_norm)
    y = MLA attention(y)                                      (wh_v4_attention)
    x = hc_post(y, residual, post, comb)                      (wh_hc_post)
    residual = x;  y, post, comb = hc_pre(hc_ffn, x)
    y = rms_norm(y, post_attention_layernorm)
    y = routed experts + shared expert(y)                     (wh_moe_ffn)
    x = hc_post(y, residual, post, comb)

and after the last layer the pooled head (hc_head_pool, final norm) and the
lm_head top-k of every sequence (wh_lm_head_topk_batch).  Every kernel is the bit-exact one, so the
step equals the oracle's composition of the same functions.

The step takes `batch` sequences, each at its own position with its own
latent KV cache per layer; the compressed rows of each layer (the DSA
compressor's output, whose feed is not part of this path) are given per
sequence.  All calls go to one stream, so a step can be captured once in a
CUDA graph and replayed (positions are fixed per captured graph).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

from . import (DEEPSEEK_V4_HC_EPS, DEEPSEEK_V4_HC_SINKHORN_ITERS, Context, MoeLayer,
               V4Attention, deepseek_rope_for_layer, hc_head, hc_post, hc_pre,
               lm_head_topk_score_batch, rms_norm, rope_inv_freqs, v4_attention,
               v4_attention_scratch_len)


@dataclass
class V4LayerWeights:
    """One layer: attention, the two norms (bf16 bits), the two mHC parameter
    sets (fn [(2+hc)*hc, hc*hidden], scale [3], base [(2+hc)*hc], f32) and the
    MoE FFN (router + routed experts + shared expert)."""
    index: int
    attn: V4Attention
    attn_norm: object
    ffn_norm: object
    hc_attn: tuple
    hc_ffn: tuple
    moe: MoeLayer


class V4Decoder:
    """The decode step of `layers` for `batch` sequences.

    kv_caches[b][l]: [positions, head_dim] f32 latent cache of sequence b,
    layer l; compressed[b][l]: [count, head_dim] f32 or None.  head:
    (fn [hc, hc*hidden], scale (float), base [hc]) of hc_head_pool; final_norm
    bf16 bits [hidden]; lm_head bf16 bits [vocab, hidden]."""

    def __init__(self, ctx: Context, layers: Sequence[V4LayerWeights], head: tuple, final_norm,
                 lm_head, kv_caches, compressed, batch: int, hc: int = 4, hidden: int = 4096,
                 top_k: int = 1):
        import torch

        self.ctx = ctx
        self.layers = list(layers)
        self.head = head
        self.final_norm = final_norm
        self.lm_head = lm_head
        self.kv = kv_caches
        self.comp = compressed
        self.batch = batch
        self.hc = hc
        self.hidden = hidden
        self.top_k = top_k
        dev = lm_head.device
        B = batch
        self.resid = torch.empty(B, hc * hidden, device=dev)
        self.x2 = torch.empty(B, hc * hidden, device=dev)
        self.y = torch.empty(B, hidden, device=dev)
        self.y2 = torch.empty(B, hidden, device=dev)
        self.post = torch.empty(B, hc, device=dev)
        self.comb = torch.empty(B, hc, hc, device=dev)
        self.pooled = torch.empty(B, hidden, device=dev)
        n = max(v4_attention_scratch_len(L.attn, B) for L in self.layers)
        self.attn_scratch = torch.empty(n, device=dev)
        self.freqs = [rope_inv_freqs(L.attn.head_dim - L.attn.nope_dim,
                                     *deepseek_rope_for_layer(L.index)) for L in self.layers]
        self.tokens = torch.empty(B, max(top_k, 1), dtype=torch.int32, device=dev)
        self.logits = torch.empty(B, max(top_k, 1), device=dev)
        from . import lib

        self.lm_scratch = torch.empty(lib().wh_lm_head_batch_scratch_bytes(
            lm_head.shape[0], max(top_k, 1), B), dtype=torch.uint8, device=dev)

    def step(self, x, positions: Sequence[int]):
        """One decode position per sequence: x [batch, hc*hidden] is the
        residual stream entering layer 0 (updated in place); returns the
        top-k token ids and logits per sequence (device tensors)."""
        hc, H = self.hc, self.hidden
        c = self.ctx
        for li, L in enumerate(self.layers):
            # --- attention sub-block (phase 1) ---
            self.resid.copy_(x)
            fn, scale, base = L.hc_attn
            hc_pre(c, fn, scale, base, x, hc, H, DEEPSEEK_V4_HC_SINKHORN_ITERS,
                   DEEPSEEK_V4_HC_EPS, out=(self.y, self.post, self.comb))
            rms_norm(c, self.y, L.attn_norm, out=self.y)
            v4_attention(c, L.attn, list(positions), self.y,
                         [self.kv[b][li] for b in range(self.batch)], self.freqs[li],
                         [self.comp[b][li] for b in range(self.batch)], self.attn_scratch)
            hc_post(c, self.y, self.resid, self.post, self.comb, hc, H, out=x)
            # --- ffn hc_pre + norm (phase 1), MoE + hc_post (phase 2) ---
            self.resid.copy_(x)
            fn, scale, base = L.hc_ffn
            hc_pre(c, fn, scale, base, x, hc, H, DEEPSEEK_V4_HC_SINKHORN_ITERS,
                   DEEPSEEK_V4_HC_EPS, out=(self.y, self.post, self.comb))
            rms_norm(c, self.y, L.ffn_norm, out=self.y)
            L.moe.forward(self.y, self.y2)
            hc_post(c, self.y2, self.resid, self.post, self.comb, hc, H, out=x)
        fn, scale, base = self.head
        hc_head(c, fn, scale, base, x, hc, H, DEEPSEEK_V4_HC_EPS, out=self.pooled)
        rms_norm(c, self.pooled, self.final_norm, out=self.pooled)
        # every sequence's lm_head top-k in one call: the 129280 x 4096 weight
        # streams once per tile of 8 sequences, not once per sequence
        t, v = lm_head_topk_score_batch(c, self.lm_head, self.pooled, self.top_k,
                                        scratch=self.lm_scratch)
        self.tokens[:, :t.shape[1]].copy_(t)
        self.logits[:, :v.shape[1]].copy_(v)
        return self.tokens, self.logits
