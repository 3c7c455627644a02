"""CPU restatement of the Qwen3 decoder in the device decoder's fixed order. TEST INFRASTRUCTURE ONLY.

Follows the reference's model stack step by step:

- embedding lookup (src/models/qwen3/qwen3_model.cpp:132-165), then per layer
  (src/nn/qwen_decoder_block.cpp:65-90):
  - ops::rms_norm with input_layernorm (nn_ops.cpp:140-201);
  - q/k/v projections (src/nn/qwen_attention.cpp:346-351, linear_project src/nn/qwen_common.cpp:15-37);
  - per-head q/k RMSNorm and RoPE at the cached positions (qwen_attention.cpp:383-390);
  - K/V appended to the cache (src/nn/qwen_cache.cpp:141-234);
  - causal GQA attention with bf16 probabilities (qwen_attention.cpp:236-333);
  - o_proj, residual add, post_attention_layernorm, the gated MLP (src/nn/qwen_mlp.cpp:55-72), residual add;
- the final norm and the tied-embedding LM head (qwen3_model.cpp:301-311);
- greedy selection (src/cli/cli_app.cpp:72-94).

Every elementwise op, norm and RoPE is the bit-exact restatement in oracle/oracle.c; the projections, the attention
and the exp inside SiLU and softmax use the fixed orders documented there (oracle_linear_canonical,
oracle_decoder_attention, oracle_pexp). bf16 tensors are numpy uint16 bit patterns.
"""

from __future__ import annotations

import numpy as np

from .oracle import Oracle


class OracleQwen3:
    """A Qwen3 model with one cached sequence (batch 1), computed on the CPU."""

    def __init__(self, config, weights: dict, max_sequence_length: int, oracle: Oracle | None = None):
        self.cfg = config
        self.w = weights
        self.o = oracle or Oracle()
        self.cap = int(max_sequence_length)
        c = config
        self.k_cache = [np.zeros((self.cap, c.num_key_value_heads, c.head_dim), np.uint16)
                        for _ in range(c.num_hidden_layers)]
        self.v_cache = [np.zeros_like(k) for k in self.k_cache]
        self.length = 0

    def reset(self) -> None:
        for k, v in zip(self.k_cache, self.v_cache):
            k.fill(0)
            v.fill(0)
        self.length = 0

    def _layer(self, i: int, h: np.ndarray, pos0: int) -> np.ndarray:
        c, o, w = self.cfg, self.o, self.w
        p = f"model.layers.{i}."
        t = h.shape[0]
        xn = o.rms_norm(h, w[p + "input_layernorm.weight"], c.rms_norm_eps)
        q = o.linear_canonical(xn, w[p + "self_attn.q_proj.weight"])
        k = o.linear_canonical(xn, w[p + "self_attn.k_proj.weight"])
        v = o.linear_canonical(xn, w[p + "self_attn.v_proj.weight"])
        q = q.reshape(t, c.num_attention_heads, c.head_dim)
        k = k.reshape(t, c.num_key_value_heads, c.head_dim)
        qr, kr = o.qk_norm_rope(q, k, w[p + "self_attn.q_norm.weight"], w[p + "self_attn.k_norm.weight"],
                                c.rms_norm_eps, offset=pos0, base=c.rope_theta)
        self.k_cache[i][pos0:pos0 + t] = kr
        self.v_cache[i][pos0:pos0 + t] = v.reshape(t, c.num_key_value_heads, c.head_dim)
        ctx = o.decoder_attention(qr, self.k_cache[i], self.v_cache[i], pos0)
        attn = o.linear_canonical(ctx.reshape(t, -1), w[p + "self_attn.o_proj.weight"])
        h1 = o.add(h, attn)
        xn2 = o.rms_norm(h1, w[p + "post_attention_layernorm.weight"], c.rms_norm_eps)
        g = o.linear_canonical(xn2, w[p + "mlp.gate_proj.weight"])
        u = o.linear_canonical(xn2, w[p + "mlp.up_proj.weight"])
        m = o.silu_mul_pexp(g, u)
        d = o.linear_canonical(m, w[p + "mlp.down_proj.weight"])
        return o.add(h1, d)

    def forward_cached(self, token_ids, all_logits: bool = False) -> np.ndarray:
        """Appends `token_ids` to the cached sequence; returns bf16 logits [T, vocab] (or [1, vocab], the last row)."""
        ids = np.asarray(token_ids, dtype=np.int64)
        c = self.cfg
        if ids.ndim != 1 or ids.size == 0:
            raise ValueError("forward_cached requires a non-empty 1-D token id list.")
        if self.length + ids.size > self.cap:
            raise ValueError("forward_cached would overflow the cache.")
        if ids.min() < 0 or ids.max() >= c.vocab_size:
            raise IndexError("Qwen3Model token id is out of vocabulary range.")
        embed = self.w["model.embed_tokens.weight"]
        h = np.ascontiguousarray(embed[ids])
        pos0 = self.length
        for i in range(c.num_hidden_layers):
            h = self._layer(i, h, pos0)
        self.length += ids.size
        rows = h if all_logits else h[-1:]
        xf = self.o.rms_norm(np.ascontiguousarray(rows), self.w["model.norm.weight"], c.rms_norm_eps)
        return self.o.linear_canonical(xf, embed)

    def generate(self, prompt, steps: int) -> list[int]:
        """Greedy decoding: prefill `prompt`, then `steps` tokens, each the argmax of the last logits row."""
        logits = self.forward_cached(prompt)
        out = [int(self.o.row_argmax(logits)[0])]
        for _ in range(steps - 1):
            logits = self.forward_cached([out[-1]])
            out.append(int(self.o.row_argmax(logits)[0]))
        return out
