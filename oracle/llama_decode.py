"""CPU oracle for the GGUF decode step — TEST INFRASTRUCTURE ONLY.

Only tests/ may import this module; the product never calls it.

It restates, in numpy, the reference's CPU executor for llama-family GGUF
models (sadrasa97/DracoRT, paths relative to that project), operation by
operation in the same fp32 / float64 order:

* ``config_from_metadata`` — the llama branch of GGUFReader's metadata
  mapping, draco/format/gguf.py:680-770 (hidden size, layers, heads, key/value
  heads, vocab, rope_theta, rms epsilon, tied embeddings);
* ``rms_norm``, ``swiglu``, ``build_rope_cache``, ``apply_rope``, ``softmax`` —
  draco/runtime/cpu/ops.py:15-27, 68-95;
* ``OracleLlama.forward_step`` — CPUExecutionBackend.forward_step,
  draco/runtime/cpu/executor.py:282-341 (embedding gather, per layer
  RMSNorm -> q/k/v -> RoPE -> cached causal attention -> o_proj -> residual,
  RMSNorm -> gate/up -> SwiGLU -> down -> residual, final norm, lm_head or
  tied embedding);
* ``OracleLlama.forward_batch_decode`` — executor.py:343-396;
* the attention — CPUAttentionBackend.prefill / decode,
  draco/runtime/cpu/attention.py (append k / v, then
  softmax(q K^T * (1 / sqrt(d))) V, causal mask for prefill; the scale is a
  numpy float64 scalar, so the scores and the softmax are float64 there);
* every linear layer — executor._linear (executor.py:47-79) on weights
  dequantized by gguf_oracle.dequantize, i.e. matmul_f32 (x @ W.T in fp32);
* ``layer_decode_step`` / ``layer_decode_batch`` / ``head_step`` — the same
  per-layer body (one new token; or one token for each of n sequences, as
  forward_batch_decode) and head over contiguous cache arrays (the reference's
  CPUKVCache.get returns the rows contiguous; attention.py:36-74), the form
  the CPU baseline of the decode-step benchmark times.

The GGUF container is parsed with dracort_b200.format.gguf_file (checked on
its own against the reference reader's index); only the arithmetic is
restated here.  Pinning: tests/golden/tiny_llama_decode_ref.npz holds the
reference executor's logits for tests/golden/tiny_llama_decode.gguf
(tests/golden/make_decode_golden.py), and test_decode_oracle.py checks this
module against them.
"""

from __future__ import annotations

from typing import Dict, List

import numpy as np

from oracle import gguf_oracle as O

_BLOCK_NAMES = {
    "attn_norm.weight": "input_layernorm.weight",
    "attn_q.weight": "q_proj",
    "attn_k.weight": "k_proj",
    "attn_v.weight": "v_proj",
    "attn_output.weight": "o_proj",
    "ffn_norm.weight": "post_attention_layernorm.weight",
    "ffn_gate.weight": "gate_proj",
    "ffn_up.weight": "up_proj",
    "ffn_down.weight": "down_proj",
}


def config_from_metadata(meta: Dict, tensor_names) -> Dict:
    """gguf.py:680-770, llama branch (the flags of gguf.py:765-768 tested on
    layer 0's tensors under their GGUF names)."""
    arch = meta.get("general.architecture", "llama")
    p = arch + "."
    hidden = int(meta[p + "embedding_length"])
    heads = int(meta[p + "attention.head_count"])
    kv_heads = int(meta.get(p + "attention.head_count_kv") or heads)
    vocab = meta.get(p + "vocab_size")
    if vocab is None:
        vocab = None  # taken from the embedding shape by the caller
    rms = meta.get(p + "attention.layer_norm_rms_epsilon") or meta.get(p + "attention.layer_norm_epsilon") or 1e-5
    has_output = "output.weight" in tensor_names
    return {
        "hidden_size": hidden,
        "num_hidden_layers": int(meta[p + "block_count"]),
        "num_attention_heads": heads,
        "num_key_value_heads": kv_heads,
        "vocab_size": vocab,
        "max_position_embeddings": int(meta.get(p + "context_length") or 4096),
        "rope_theta": float(meta.get(p + "rope.freq_base", 10000.0)),
        "qkv_fused": "blk.0.attn_qkv.weight" in tensor_names,
        "attention_bias": "blk.0.attn_q.bias" in tensor_names,
        "mlp_bias": "blk.0.ffn_gate.bias" in tensor_names,
        "rms_norm_eps": float(rms),
        "tie_word_embeddings": bool(meta.get(p + "tie_embeddings", not has_output)),
    }


def rms_norm(x, weight, eps):
    x32 = x.astype(np.float32)
    variance = np.mean(x32 * x32, axis=-1, keepdims=True)
    normed = x32 / np.sqrt(variance + eps)
    return (normed * weight).astype(x.dtype)


def swiglu(gate, up):
    return gate * (1.0 / (1.0 + np.exp(-gate))) * up


def softmax(x, axis=-1):
    x = x - np.max(x, axis=axis, keepdims=True)
    e = np.exp(x)
    return e / np.sum(e, axis=axis, keepdims=True)


def build_rope_cache(head_dim, max_positions, theta):
    inv_freq = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    positions = np.arange(max_positions, dtype=np.float32)
    freqs = np.outer(positions, inv_freq)
    return np.cos(freqs), np.sin(freqs)


def apply_rope(x, cos, sin, positions):
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c = cos[positions][:, None, :]
    s = sin[positions][:, None, :]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(x.dtype)


class OracleLlama:
    """CPUExecutionBackend restated for one GGUF file (q6k_order: byte order of
    the file's Q6_K blocks, "d_first" as the reference decodes them)."""

    def __init__(self, gguf_file, q6k_order: str = "d_first") -> None:
        gf = gguf_file
        self.cfg = cfg = config_from_metadata(gf.metadata, gf.tensors)
        self.w: Dict[str, np.ndarray] = {}
        for name, t in gf.tensors.items():
            payload = np.asarray(gf.payload(name)).reshape(-1)
            if t.is_quantized:
                arr = O.dequantize(t.ggml_type, payload, int(np.prod(t.shape)), q6k_order=q6k_order)
            elif t.ggml_type == 1:
                arr = payload.view(np.float16).astype(np.float32)
            else:
                arr = payload.view(np.float32).astype(np.float32)
            self.w[name] = arr.reshape(t.shape)
        if cfg["vocab_size"] is None:
            cfg["vocab_size"] = self.w["token_embd.weight"].shape[0]
        self.head_dim = cfg["hidden_size"] // cfg["num_attention_heads"]
        self.cos, self.sin = build_rope_cache(self.head_dim, cfg["max_position_embeddings"], cfg["rope_theta"])
        self.group = cfg["num_attention_heads"] // cfg["num_key_value_heads"]
        self.kv: Dict[int, List[List[np.ndarray]]] = {}  # seq -> layer -> [k list, v list]
        self._next = 0

    # -- sequences (executor.py:172-183) --------------------------------------
    def new_sequence(self) -> int:
        s = self._next
        self._next += 1
        self.kv[s] = [[[], []] for _ in range(self.cfg["num_hidden_layers"])]
        return s

    def end_sequence(self, s: int) -> None:
        self.kv.pop(s, None)

    def _linear(self, name, x, bias=None):
        """executor._linear (executor.py:47-79): matmul_f32, then `+ bias` when
        the bias tensor exists."""
        out = x.astype(np.float32, copy=False) @ self.w[name].astype(np.float32, copy=False).T
        if bias is not None and bias in self.w:
            out = out + self.w[bias]
        return out

    def _attention(self, s, layer, q, k, v, causal):
        """attention.py prefill: append, then attend over the whole cache."""
        ks, vs = self.kv[s][layer]
        for t in range(q.shape[0]):
            ks.append(k[t])
            vs.append(v[t])
        ck = np.repeat(np.stack(ks).astype(np.float32), self.group, axis=1)
        cv = np.repeat(np.stack(vs).astype(np.float32), self.group, axis=1)
        scale = 1.0 / np.sqrt(q.shape[-1])
        q_t = np.transpose(q.astype(np.float32), (1, 0, 2))
        k_t = np.transpose(ck, (1, 0, 2))
        v_t = np.transpose(cv, (1, 0, 2))
        scores = np.einsum("hqd,hkd->hqk", q_t, k_t) * scale
        if causal:
            total = k_t.shape[1]
            qpos = np.arange(total - q.shape[0], total)
            mask = np.arange(total)[None, :] > qpos[:, None]
            scores = np.where(mask[None, :, :], -np.inf, scores)
        out = np.einsum("hqk,hkd->hqd", softmax(scores, axis=-1), v_t)
        return np.transpose(out, (1, 0, 2)).astype(q.dtype)

    def _layer_qkv(self, layer, hidden, n):
        """executor.py:243-271.  A fused q/k/v weight is split by columns of its
        output; its bias is looked up under the GPT-2 name there, which a
        llama-family file never has, so none is added."""
        cfg, p = self.cfg, f"blk.{layer}."
        heads, kvh, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], self.head_dim
        normed = rms_norm(hidden, self.w[p + "attn_norm.weight"], cfg["rms_norm_eps"])
        if cfg["qkv_fused"]:
            qkv = self._linear(p + "attn_qkv.weight", normed)
            q, k, v = qkv[:, :heads * hd], qkv[:, heads * hd:(heads + kvh) * hd], qkv[:, (heads + kvh) * hd:]
        else:
            b = cfg["attention_bias"]
            q = self._linear(p + "attn_q.weight", normed, p + "attn_q.bias" if b else None)
            k = self._linear(p + "attn_k.weight", normed, p + "attn_k.bias" if b else None)
            v = self._linear(p + "attn_v.weight", normed, p + "attn_v.bias" if b else None)
        return q.reshape(n, heads, hd), k.reshape(n, kvh, hd), v.reshape(n, kvh, hd)

    def _layer_rest(self, layer, hidden, attn_out):
        """o_proj (executor.py:273-277, its bias under attention_bias) and the
        gated MLP (executor.py:208-224, biases under mlp_bias)."""
        cfg, p = self.cfg, f"blk.{layer}."
        ab, mb = cfg["attention_bias"], cfg["mlp_bias"]
        hidden = hidden + self._linear(p + "attn_output.weight", attn_out, p + "attn_output.bias" if ab else None)
        normed = rms_norm(hidden, self.w[p + "ffn_norm.weight"], cfg["rms_norm_eps"])
        gate = self._linear(p + "ffn_gate.weight", normed, p + "ffn_gate.bias" if mb else None)
        up = self._linear(p + "ffn_up.weight", normed, p + "ffn_up.bias" if mb else None)
        return hidden + self._linear(p + "ffn_down.weight", swiglu(gate, up), p + "ffn_down.bias" if mb else None)

    def _head(self, hidden):
        cfg = self.cfg
        hidden = rms_norm(hidden, self.w["output_norm.weight"], cfg["rms_norm_eps"])
        if cfg["tie_word_embeddings"]:
            return hidden @ self.w["token_embd.weight"].T
        return self._linear("output.weight", hidden)

    def forward_step(self, s, token_ids, start_position, return_all_positions=False):
        """executor.py:282-341."""
        cfg = self.cfg
        n = len(token_ids)
        positions = np.arange(start_position, start_position + n)
        hidden = self.w["token_embd.weight"][np.asarray(token_ids)].astype(np.float32)
        for layer in range(cfg["num_hidden_layers"]):
            q, k, v = self._layer_qkv(layer, hidden, n)
            q = apply_rope(q, self.cos, self.sin, positions)
            k = apply_rope(k, self.cos, self.sin, positions)
            attn = self._attention(s, layer, q, k, v, causal=True).reshape(n, -1)
            hidden = self._layer_rest(layer, hidden, attn)
        logits = self._head(hidden)
        return logits if return_all_positions else logits[-1]

    def forward_batch_decode(self, seq_ids, token_ids, positions):
        """executor.py:343-396 (one token per sequence)."""
        cfg = self.cfg
        n = len(seq_ids)
        pos = np.array(positions)
        hidden = self.w["token_embd.weight"][np.array(token_ids)].astype(np.float32)
        for layer in range(cfg["num_hidden_layers"]):
            q, k, v = self._layer_qkv(layer, hidden, n)
            attn = np.empty((n, cfg["num_attention_heads"], self.head_dim), dtype=np.float32)
            for i in range(n):
                qi = apply_rope(q[i:i + 1], self.cos, self.sin, pos[i:i + 1])
                ki = apply_rope(k[i:i + 1], self.cos, self.sin, pos[i:i + 1])
                attn[i] = self._attention(seq_ids[i], layer, qi, ki, v[i:i + 1], causal=False)[0]
            hidden = self._layer_rest(layer, hidden, attn.reshape(n, -1))
        return self._head(hidden)


def _mm(x, w):
    """executor._linear's matmul_f32: x @ W.T in fp32."""
    return x.astype(np.float32, copy=False) @ w.astype(np.float32, copy=False).T


def layer_decode_step(hidden, w, k_cache, v_cache, length, cos, sin, eps, heads, kv_heads):
    """One decoder layer of forward_step for one new token (executor.py:282-341,
    the loop body), attention as CPUAttentionBackend.prefill / decode computes
    it (attention.py:36-74: append, gather rows 0..length, fp32 cast, GQA
    repeat, float64 scores through the float64 scale, softmax, weighted sum).

    hidden [1, H] fp32; w: fp32 arrays "attn_norm", "q", "k", "v", "o",
    "ffn_norm", "gate", "up", "down" (projections [out, in]); k_cache /
    v_cache [capacity, kv_heads, head_dim] holding `length` rows, the token's
    key and value written to row `length`.  Returns the layer's output."""
    hd = hidden.shape[-1] // heads
    normed = rms_norm(hidden, w["attn_norm"], eps)
    q = _mm(normed, w["q"]).reshape(1, heads, hd)
    k = _mm(normed, w["k"]).reshape(1, kv_heads, hd)
    v = _mm(normed, w["v"]).reshape(1, kv_heads, hd)
    pos = np.array([length])
    q = apply_rope(q, cos, sin, pos)
    k = apply_rope(k, cos, sin, pos)
    k_cache[length] = k[0]
    v_cache[length] = v[0]
    group = heads // kv_heads
    ck = np.repeat(k_cache[:length + 1].astype(np.float32), group, axis=1)
    cv = np.repeat(v_cache[:length + 1].astype(np.float32), group, axis=1)
    scale = 1.0 / np.sqrt(hd)
    q_t = np.transpose(q.astype(np.float32), (1, 0, 2))
    scores = np.einsum("hqd,hkd->hqk", q_t, np.transpose(ck, (1, 0, 2))) * scale
    out = np.einsum("hqk,hkd->hqd", softmax(scores, axis=-1), np.transpose(cv, (1, 0, 2)))
    attn = np.transpose(out, (1, 0, 2)).astype(np.float32).reshape(1, -1)
    hidden = hidden + _mm(attn, w["o"])
    normed = rms_norm(hidden, w["ffn_norm"], eps)
    return hidden + _mm(swiglu(_mm(normed, w["gate"]), _mm(normed, w["up"])), w["down"])


def layer_decode_batch(hidden, w, caches, lengths, cos, sin, eps, heads, kv_heads):
    """One decoder layer of forward_batch_decode (executor.py:343-396): the
    projections over all n rows at once, RoPE and the attention per sequence
    (row i over caches[i] = (k_cache, v_cache) holding lengths[i] rows, its
    key and value written to row lengths[i]), then o_proj and the MLP over
    all rows.  hidden [n, H] fp32."""
    n = hidden.shape[0]
    hd = hidden.shape[-1] // heads
    normed = rms_norm(hidden, w["attn_norm"], eps)
    q = _mm(normed, w["q"]).reshape(n, heads, hd)
    k = _mm(normed, w["k"]).reshape(n, kv_heads, hd)
    v = _mm(normed, w["v"]).reshape(n, kv_heads, hd)
    group = heads // kv_heads
    scale = 1.0 / np.sqrt(hd)
    attn = np.empty((n, heads, hd), dtype=np.float32)
    for i in range(n):
        length = int(lengths[i])
        kc, vc = caches[i]
        qi = apply_rope(q[i:i + 1], cos, sin, np.array([length]))
        ki = apply_rope(k[i:i + 1], cos, sin, np.array([length]))
        kc[length] = ki[0]
        vc[length] = v[i]
        ck = np.repeat(kc[:length + 1].astype(np.float32), group, axis=1)
        cv = np.repeat(vc[:length + 1].astype(np.float32), group, axis=1)
        scores = np.einsum("hqd,hkd->hqk", np.transpose(qi, (1, 0, 2)), np.transpose(ck, (1, 0, 2))) * scale
        o = np.einsum("hqk,hkd->hqd", softmax(scores, axis=-1), np.transpose(cv, (1, 0, 2)))
        attn[i] = np.transpose(o, (1, 0, 2))[0]
    hidden = hidden + _mm(attn.reshape(n, -1), w["o"])
    normed = rms_norm(hidden, w["ffn_norm"], eps)
    return hidden + _mm(swiglu(_mm(normed, w["gate"]), _mm(normed, w["up"])), w["down"])


def head_step(hidden, norm_w, w_out, eps):
    """The final RMSNorm and the output projection (executor.py:330-341)."""
    return _mm(rms_norm(hidden, norm_w, eps), w_out)
