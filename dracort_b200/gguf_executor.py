"""GPU decode step for llama-family GGUF models: a drop-in for the reference's
``CPUExecutionBackend`` (draco/runtime/cpu/executor.py:132-413) on the GGUF
path, where ``LLM._generate_single_gguf`` (draco/engine/llm.py:1158-1199)
drives it through ``new_sequence`` / ``forward_step`` / ``end_sequence``.

The reference dequantizes every weight to an fp32 cache on the host and runs
numpy.  Here the whole step runs on one GPU:

* weights stay packed (the TILED layout of ``gguf_loader.load_gguf``); each
  layer takes four GEMV steps — q/k/v with the attention RMSNorm fused into
  the activation read, o_proj adding into the hidden state, gate/up with the
  MLP RMSNorm fused, down reading the SwiGLU product and adding into the
  hidden state — and the output head reads the final RMSNorm the same way;
  dense (F16 / F32) projections of a file go through an fp32 matmul instead;
* RoPE (rotate-half, draco/runtime/cpu/ops.py:77-95), the key/value-cache
  append and the causal attention over the cache
  (draco/runtime/cpu/attention.py; fp32, grouped-query heads) run as one
  kernel, ``draco_attention_decode``, when a pass's tokens hold distinct
  slots (decode steps), and as ``draco_rope_kv_append`` +
  ``draco_attention_cached`` for a prompt;
* each pass is recorded once as a CUDA graph per (rows, attention bound,
  form) and replayed, over fixed buffers, with the residual adds folded into
  the o_proj / down GEMVs (DRACO_GEMV_ACCUMULATE);
* the key/value cache is a per-layer fp32 tensor [slot, kv_heads, capacity,
  head_dim]: a sequence owns one slot from ``new_sequence`` to
  ``end_sequence``.

Rows go through the GEMV 32 at a time, so prompts are processed in chunks
of 32 tokens (each chunk attends to everything cached before it).  Results
follow the decode GEMV's accuracy (about 1e-4 relative L2 per projection
against the fp32 reference); ``forward_step`` / ``forward_batch_decode``
return numpy fp32 logits like the reference.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from dracort_b200 import _native as N
from dracort_b200 import gguf_ops as G
from dracort_b200.exceptions import DracoFormatError
from dracort_b200.format.gguf_file import GGUFFile
from dracort_b200.format.gguf_types import BLOCK_LAYOUTS, GGML_TYPE_Q6_K, Q6K_D_LAST
from dracort_b200.gguf_loader import DeviceWeight, load_gguf

_ROWS = N.GEMV_MAX_BATCH  # activation rows per GEMV call


@dataclass
class LlamaConfig:
    """The llama-family configuration the reference derives from GGUF metadata
    (draco/format/gguf.py:680-770)."""

    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    vocab_size: int
    max_position_embeddings: int
    rope_theta: float
    rms_norm_eps: float
    tie_word_embeddings: bool
    qkv_fused: bool = False       # one attn_qkv weight per layer (q rows, then k, then v)
    attention_bias: bool = False  # q/k/v (unfused) and o_proj biases where the file has them
    mlp_bias: bool = False        # gate/up/down biases where the file has them

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @classmethod
    def from_gguf(cls, gf: GGUFFile) -> "LlamaConfig":
        meta = gf.metadata
        arch = str(meta.get("general.architecture", "llama"))
        if arch == "gpt2":
            raise DracoFormatError("the GPU decode step runs llama-family GGUF models (gpt2 is not supported)")
        p = arch + "."

        def get(key, default=None):
            v = meta.get(p + key)
            return default if v is None else v

        hidden, layers, heads = get("embedding_length"), get("block_count"), get("attention.head_count")
        vocab = get("vocab_size")
        if vocab is None and "token_embd.weight" in gf.tensors:
            vocab = gf.tensor("token_embd.weight").shape[0]
        if None in (hidden, layers, heads, vocab):
            missing = [k for k, v in (("embedding_length", hidden), ("block_count", layers),
                                      ("attention.head_count", heads), ("vocab_size", vocab)) if v is None]
            raise DracoFormatError(f"{gf.path}: no {', '.join(p + k for k in missing)} in the GGUF metadata")
        key_len = get("attention.key_length")
        if key_len is not None and int(key_len) != int(hidden) // int(heads):
            raise DracoFormatError(f"{gf.path}: attention key length {key_len} differs from "
                                   f"embedding_length / head_count = {int(hidden) // int(heads)}")
        eps = get("attention.layer_norm_rms_epsilon") or get("attention.layer_norm_epsilon") or 1e-5
        return cls(hidden_size=int(hidden), num_hidden_layers=int(layers), num_attention_heads=int(heads),
                   num_key_value_heads=int(get("attention.head_count_kv") or heads), vocab_size=int(vocab),
                   max_position_embeddings=int(get("context_length") or 4096),
                   rope_theta=float(get("rope.freq_base", 10000.0)), rms_norm_eps=float(eps),
                   tie_word_embeddings=bool(get("tie_embeddings", "output.weight" not in gf.tensors)),
                   # the flags of gguf.py:765-768, from layer 0's tensors
                   qkv_fused="blk.0.attn_qkv.weight" in gf.tensors,
                   attention_bias="blk.0.attn_q.bias" in gf.tensors,
                   mlp_bias="blk.0.ffn_gate.bias" in gf.tensors)


def rope_tables(head_dim: int, max_positions: int, theta: float):
    """cos / sin [max_positions, head_dim / 2] fp32, computed on the host in the
    reference's order (build_rope_cache, draco/runtime/cpu/ops.py:77-83)."""
    inv_freq = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    freqs = np.outer(np.arange(max_positions, dtype=np.float32), inv_freq)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


_PROJ = {"q": "attn_q", "k": "attn_k", "v": "attn_v", "o": "attn_output", "gate": "ffn_gate", "up": "ffn_up",
         "down": "ffn_down"}


def layer_tensors(cfg: LlamaConfig, tensor_names, layer: int) -> Dict[str, object]:
    """The tensors behind layer `layer`, as the reference's executor picks them
    (executor.py:208-277 with the flags of gguf.py:765-768):

    "attn_norm", "ffn_norm": norm weight names;
    "proj": {q, k, v, o, gate, up, down: (tensor name, (row0, row1) or None)}
        — a fused attn_qkv weight gives q, k and v as row ranges of it;
    "bias": {projection: bias tensor name or None} — q/k/v and o_proj under
        attention_bias (none for a fused weight: the reference looks its bias
        up under the GPT-2 name, which a llama-family file never has),
        gate/up/down under mlp_bias; only biases the file has."""
    p = f"blk.{layer}."
    names = set(tensor_names)
    proj = {key: (p + stem + ".weight", None) for key, stem in _PROJ.items()}
    if cfg.qkv_fused:
        hd = cfg.head_dim
        qr, kr = cfg.num_attention_heads * hd, cfg.num_key_value_heads * hd
        fused = p + "attn_qkv.weight"
        proj["q"], proj["k"], proj["v"] = (fused, (0, qr)), (fused, (qr, qr + kr)), (fused, (qr + kr, qr + 2 * kr))
    bias = {}
    for key, stem in _PROJ.items():
        on = cfg.mlp_bias if key in ("gate", "up", "down") else cfg.attention_bias
        if key in ("q", "k", "v") and cfg.qkv_fused:
            on = False
        name = p + stem + ".bias"
        bias[key] = name if on and name in names else None
    return {"attn_norm": p + "attn_norm.weight", "ffn_norm": p + "ffn_norm.weight", "proj": proj, "bias": bias}


def _row_range_weight(gf: GGUFFile, name: str, r0: int, r1: int, device: torch.device,
                      q6k_order: str) -> DeviceWeight:
    """Rows [r0, r1) of a quantized GGUF weight, regrouped on the device (the
    rows of a GGUF weight are independent runs of blocks)."""
    t = gf.tensor(name)
    bs, bb = BLOCK_LAYOUTS[t.ggml_type]
    rows = np.ascontiguousarray(np.asarray(gf.payload(name)).reshape(t.n_rows, t.k // bs * bb)[r0:r1])
    raw = torch.from_numpy(rows.reshape(-1)).to(device)
    layout = "gguf_dlast" if (t.ggml_type == GGML_TYPE_Q6_K and q6k_order == Q6K_D_LAST) else "gguf"
    tiled = G.repack(t.ggml_type, raw, r1 - r0, t.k, layout=layout)
    return DeviceWeight(name, t.ggml_type, tiled, r1 - r0, t.k, r0, r1, 0, t.k)


def cache_capacity(cfg: LlamaConfig, max_num_seqs: int, max_seq_len: Optional[int] = None,
                   kv_budget_bytes: Optional[int] = None) -> int:
    """Cache rows per sequence: max_seq_len, else as many as kv_budget_bytes
    holds for max_num_seqs sequences (fp32 keys and values of every layer,
    the budget CPUExecutionBackend takes, executor.py:145-159), else the
    model's context length; never above the context length."""
    cap = int(cfg.max_position_embeddings)
    if max_seq_len is not None:
        cap = min(int(max_seq_len), cap)
    elif kv_budget_bytes is not None:
        per_pos = int(max_num_seqs) * cfg.num_hidden_layers * 2 * cfg.num_key_value_heads * cfg.head_dim * 4
        cap = min(int(kv_budget_bytes) // per_pos, cap)
    if cap < 1:
        raise ValueError(f"the key/value cache holds no position for {max_num_seqs} sequences "
                         f"(max_seq_len {max_seq_len}, kv_budget_bytes {kv_budget_bytes})")
    return cap


class GPUExecutionBackend:
    """``CPUExecutionBackend`` for llama-family GGUF files, on one GPU.

    Positional arguments as the reference's constructor (executor.py:133-140):

    source          : path of a .gguf file, an open GGUFFile, or any reader with
                      a ``path`` attribute (the reference's GGUFReader);
    max_num_seqs    : sequences that may hold a key/value cache at once;
    kv_cache_dtype  : "f32" (the cache is fp32, as the reference's default);
    kv_budget_bytes : sizes the cache when max_seq_len is not given;
    memory_utilization: accepted for the reference's signature; the cache is
                      sized by max_seq_len, kv_budget_bytes or the context.

    Keyword-only:

    device      : the CUDA device;
    max_seq_len : cache rows per sequence (default: from kv_budget_bytes, else
                  the model's context length);
    q6k_order   : byte order of the file's Q6_K blocks ("d_last" for llama.cpp
                  files, "d_first" for the order the reference decodes).
    """

    def __init__(self, source, max_num_seqs: int = 1, kv_cache_dtype: str = "f32",
                 kv_budget_bytes: Optional[int] = None, memory_utilization: Optional[float] = None, *,
                 device: Union[str, torch.device] = "cuda", max_seq_len: Optional[int] = None,
                 q6k_order: str = Q6K_D_LAST) -> None:
        if kv_cache_dtype not in ("f32", "fp32", "float32"):
            raise ValueError(f"kv_cache_dtype {kv_cache_dtype!r}: the GPU decode step keeps an fp32 cache")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("GPUExecutionBackend runs on a CUDA device (this library has no CPU path)")
        own = not isinstance(source, GGUFFile)
        if own and not isinstance(source, (str, os.PathLike)):
            if not hasattr(source, "path"):
                raise TypeError("source must be a path, a GGUFFile or a reader with a 'path' attribute")
            source = source.path
        gf = GGUFFile(os.fspath(source)) if own else source
        try:
            self.config = cfg = LlamaConfig.from_gguf(gf)
            plans = [layer_tensors(cfg, gf.tensors, i) for i in range(cfg.num_hidden_layers)]
            # quantized fused q/k/v weights load as three row ranges; everything else whole
            ranged = {(nm, rr) for pl in plans for nm, rr in pl["proj"].values() if rr is not None}
            by_rows = {nm for nm, _ in ranged if gf.tensor(nm).is_quantized}
            with torch.cuda.device(self.device):
                loaded = load_gguf(gf, self.device, q6k_order=q6k_order,
                                   names=[n for n in gf.tensors if n not in by_rows])
                for nm, (r0, r1) in ranged:
                    if nm in by_rows:
                        loaded[(nm, (r0, r1))] = _row_range_weight(gf, nm, r0, r1, self.device, q6k_order)
        finally:
            if own:
                gf.close()
        if cfg.num_attention_heads % cfg.num_key_value_heads or cfg.head_dim % 2:
            raise DracoFormatError("heads must be a multiple of key/value heads and head_dim even")

        def dense_f32(t):
            return t.to(torch.float32).contiguous()

        def entry(name):
            if name not in loaded:
                raise DracoFormatError(f"GGUF model has no tensor '{name}'")
            w = loaded[name]
            return w if isinstance(w, DeviceWeight) else dense_f32(w)

        emb = entry("token_embd.weight")
        if isinstance(emb, DeviceWeight):
            emb = G.dequantize(emb.qtype, emb.tiled, emb.n_rows, emb.k, layout="tiled")
        self.embed = emb  # [vocab, hidden] fp32

        def proj(name, rows):
            if rows is None:
                return entry(name)
            if (name, rows) in loaded:  # a quantized fused weight, loaded by rows
                return loaded[(name, rows)]
            return entry(name)[rows[0]:rows[1]].contiguous()  # a dense fused weight

        self.layers: List[Dict[str, object]] = []
        for pl in plans:
            L = {"attn_norm": entry(pl["attn_norm"]), "ffn_norm": entry(pl["ffn_norm"])}
            for key, (name, rows) in pl["proj"].items():
                L[key] = proj(name, rows)
                b = pl["bias"][key]
                L[key + "_bias"] = None if b is None else entry(b).reshape(-1)
            self.layers.append(L)
        self.final_norm = entry("output_norm.weight")
        self.lm_head = None if cfg.tie_word_embeddings else entry("output.weight")
        cap = cache_capacity(cfg, max_num_seqs, max_seq_len, kv_budget_bytes)
        self.capacity = cap
        cos, sin = rope_tables(cfg.head_dim, cap, cfg.rope_theta)
        self.cos = torch.from_numpy(cos).to(self.device)
        self.sin = torch.from_numpy(sin).to(self.device)
        self.max_num_seqs = int(max_num_seqs)
        shape = (self.max_num_seqs, cfg.num_key_value_heads, cap, cfg.head_dim)
        self.k_cache = [torch.zeros(shape, dtype=torch.float32, device=self.device) for _ in self.layers]
        self.v_cache = [torch.zeros(shape, dtype=torch.float32, device=self.device) for _ in self.layers]
        self._free = list(range(self.max_num_seqs))
        self._slot: Dict[int, int] = {}
        self._len: Dict[int, int] = {}
        self._next_seq_id = 0
        self._lib = N.load()
        self._bufs: Dict[int, Dict[str, object]] = {}
        self._graphs: Dict[Tuple[int, int, bool], torch.cuda.CUDAGraph] = {}
        self._eager_seen: set = set()
        #: replay a captured CUDA graph per (rows, attention bound) after its first eager pass
        self.use_graphs = True

    # -- sequences (executor.py:172-183) --------------------------------------
    def new_sequence(self) -> int:
        if not self._free:
            raise RuntimeError(f"all {self.max_num_seqs} key/value cache slots are in use")
        seq_id = self._next_seq_id
        self._next_seq_id += 1
        self._slot[seq_id] = self._free.pop(0)
        self._len[seq_id] = 0
        return seq_id

    def end_sequence(self, seq_id: int) -> None:
        slot = self._slot.pop(seq_id, None)
        self._len.pop(seq_id, None)
        if slot is not None:
            self._free.append(slot)

    def truncate_sequence(self, seq_id: int, new_length: int) -> None:
        """Forget cached positions from new_length on (the rows are rewritten
        by the next steps)."""
        if seq_id not in self._slot or not 0 <= new_length <= self._len[seq_id]:
            raise ValueError(f"cannot truncate sequence {seq_id} to {new_length}")
        self._len[seq_id] = new_length

    # -- compute --------------------------------------------------------------
    def _group(self, weights: Sequence[object], x: torch.Tensor, ys: Sequence[torch.Tensor],
               norm: Optional[torch.Tensor] = None, up: Optional[torch.Tensor] = None,
               accumulate: bool = False, biases: Optional[Sequence[Optional[torch.Tensor]]] = None
               ) -> Callable[[], None]:
        """One projection step over fixed buffers: ys[i] (+)= f(x) @ W_i^T
        (+ biases[i]) with f the RMSNorm by `norm`, silu(x) * up, or nothing.
        Packed weights go in one GemvPlan (the transform fused into the
        activation read, the bias and the add into the output write); dense
        ones through an fp32 matmul of the transformed x.  Returns a callable
        enqueuing the step on the current stream; its ``launches`` counts the
        library kernels it starts."""
        eps = self.config.rms_norm_eps
        biases = list(biases) if biases is not None else [None] * len(weights)
        probs, dense = [], []
        for w, y, bias in zip(weights, ys, biases):
            if isinstance(w, DeviceWeight):
                probs.append(G.GemvProblem(w.qtype, w.tiled, x, y, w.n_rows, w.k, bias=bias, norm_weight=norm,
                                           norm_eps=eps, up=up, accumulate=accumulate))
            else:
                dense.append((w, y, bias))
        plans = [G.GemvPlan(probs[i:i + N.GEMV_MAX_PROBLEMS]) for i in range(0, len(probs), N.GEMV_MAX_PROBLEMS)]

        def run() -> None:
            for pl in plans:
                pl.run()
            if dense:
                if norm is not None:
                    xd = G.rms_norm(x, norm, eps)
                elif up is not None:
                    xd = x * torch.sigmoid(x) * up
                else:
                    xd = x
                for w, y, bias in dense:
                    if accumulate:
                        y.addmm_(xd, w.t())
                    else:
                        torch.matmul(xd, w.t(), out=y)
                    if bias is not None:
                        y.add_(bias)

        run.launches = sum(pl.launches for pl in plans)  # type: ignore[attr-defined]
        return run

    def _buffers(self, n: int) -> Dict[str, object]:
        """Fixed device buffers and GEMV plans of a pass over n rows (built on
        first use, kept for the backend's lifetime)."""
        b = self._bufs.get(n)
        if b is not None:
            return b
        cfg, dev = self.config, self.device
        hd, heads, kvh = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads

        def f32(*shape):
            return torch.zeros(shape, dtype=torch.float32, device=dev)

        g0 = self.layers[0]["gate"]
        ffn = g0.n_rows if isinstance(g0, DeviceWeight) else g0.shape[0]

        b = {"ids": torch.zeros((3, n), dtype=torch.int64, device=dev),  # token, slot, position
             "stage": torch.zeros((3, n), dtype=torch.int64).pin_memory(),
             "seq": torch.zeros(n, dtype=torch.int32, device=dev),
             "pos": torch.zeros(n, dtype=torch.int32, device=dev),
             "hidden": f32(n, cfg.hidden_size), "q": f32(n, heads * hd), "k": f32(n, kvh * hd),
             "v": f32(n, kvh * hd), "attn": f32(n, heads * hd), "gate": f32(n, ffn),
             "up": f32(n, ffn), "logits": f32(n, cfg.vocab_size), "normed": f32(n, cfg.hidden_size),
             "copied": torch.cuda.Event()}
        ws_bytes = self._lib.draco_attention_workspace_bytes(n, heads, hd, self.capacity - 1)
        b["attn_ws"] = torch.zeros(int(ws_bytes), dtype=torch.uint8, device=dev)
        h = b["hidden"]
        b["layers"] = [
            (self._group([L["q"], L["k"], L["v"]], h, [b["q"], b["k"], b["v"]], norm=L["attn_norm"],
                         biases=[L["q_bias"], L["k_bias"], L["v_bias"]]),
             self._group([L["o"]], b["attn"], [h], accumulate=True, biases=[L["o_bias"]]),
             self._group([L["gate"], L["up"]], h, [b["gate"], b["up"]], norm=L["ffn_norm"],
                         biases=[L["gate_bias"], L["up_bias"]]),
             self._group([L["down"]], b["gate"], [h], up=b["up"], accumulate=True, biases=[L["down_bias"]]))
            for L in self.layers]
        b["head"] = (self._group([self.lm_head], h, [b["logits"]], norm=self.final_norm)
                     if self.lm_head is not None else None)
        self._bufs[n] = b
        return b

    @property
    def launches_per_layer(self) -> int:
        """Library kernels one decode token (a pass of one row) starts per
        layer: the four GEMV steps plus the attention."""
        return sum(g.launches for g in self._buffers(1)["layers"][0]) + 1

    def _run(self, n: int, b: Dict[str, object], max_pos: int, decode: bool) -> None:
        """Enqueue one pass of the n staged rows on the current stream (decode:
        the rows hold distinct cache slots, so that RoPE, the cache append and
        the attention run as one kernel per layer)."""
        cfg = self.config
        hd, heads, kvh = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        ids = b["ids"]
        b["seq"].copy_(ids[1])
        b["pos"].copy_(ids[2])
        torch.index_select(self.embed, 0, ids[0], out=b["hidden"])
        stream = G._stream_ptr(self.device)
        q, k, v, attn, ws = b["q"], b["k"], b["v"], b["attn"], b["attn_ws"]
        seq, pos = b["seq"].data_ptr(), b["pos"].data_ptr()
        for li, (qkv, o_proj, gate_up, down) in enumerate(b["layers"]):
            qkv()
            kc, vc = self.k_cache[li], self.v_cache[li]
            if decode:
                N.check(self._lib.draco_attention_decode(
                    q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(), self.cos.data_ptr(),
                    self.sin.data_ptr(), seq, pos, max_pos, attn.data_ptr(), n, heads, kvh, hd, self.capacity,
                    self.max_num_seqs, ws.data_ptr(), ws.numel(), stream), "attention_decode")
                o_proj()
                gate_up()
                down()
                continue
            N.check(self._lib.draco_rope_kv_append(q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(),
                                                   vc.data_ptr(), self.cos.data_ptr(), self.sin.data_ptr(), seq, pos,
                                                   n, heads, kvh, hd, self.capacity, self.max_num_seqs, stream),
                    "rope_kv_append")
            N.check(self._lib.draco_attention_cached(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), seq, pos, max_pos,
                                                     attn.data_ptr(), n, heads, kvh, hd, self.capacity,
                                                     self.max_num_seqs, ws.data_ptr(), ws.numel(), stream),
                    "attention_cached")
            o_proj()   # hidden += attn @ Wo^T
            gate_up()
            down()     # hidden += (silu(gate) * up) @ Wdown^T
        if b["head"] is not None:
            b["head"]()
        else:
            # tied embeddings (executor.py:333-334): the final norm, then x @ embed^T
            G.rms_norm(b["hidden"], self.final_norm, cfg.rms_norm_eps, out=b["normed"])
            torch.matmul(b["normed"], self.embed.t(), out=b["logits"])

    def _forward(self, slots: Sequence[int], tokens: Sequence[int], positions: Sequence[int]) -> torch.Tensor:
        """One pass of n <= 32 tokens (token i of cache slot slots[i] at
        positions[i]) through every layer; returns logits [n, vocab] fp32 in a
        buffer that the next pass over n rows overwrites.

        The attention covers positions up to a power-of-two bound of the
        largest one (at least 64, at most the capacity), so that one CUDA
        graph per (n, bound) replays every step: the first pass of a key runs
        eagerly, the second captures the graph, later ones replay it."""
        n = len(tokens)
        b = self._buffers(n)
        b["copied"].synchronize()  # the previous upload from the staging buffer has finished
        st = b["stage"]
        st[0, :] = torch.as_tensor(list(tokens), dtype=torch.int64)
        st[1, :] = torch.as_tensor(list(slots), dtype=torch.int64)
        st[2, :] = torch.as_tensor(list(positions), dtype=torch.int64)
        b["ids"].copy_(st, non_blocking=True)
        b["copied"].record()
        need = int(max(positions)) + 1
        bound = min(self.capacity, max(64, 1 << (need - 1).bit_length()))
        decode = len(set(slots)) == n
        key = (n, bound, decode)
        g = self._graphs.get(key)
        if g is not None:
            g.replay()
        elif not self.use_graphs or key not in self._eager_seen:
            self._eager_seen.add(key)
            self._run(n, b, bound - 1, decode)
        else:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._run(n, b, bound - 1, decode)
            self._graphs[key] = g
            g.replay()
        return b["logits"]

    def _check_tokens(self, tokens: Sequence[int]) -> None:
        for t in tokens:
            if not 0 <= int(t) < self.config.vocab_size:
                raise ValueError(f"token id {t} outside the vocabulary of {self.config.vocab_size}")

    def forward_step(self, seq_id: int, token_ids, start_position: int,
                     return_all_positions: bool = False) -> np.ndarray:
        """token_ids (seq_len,) of sequence seq_id from start_position (the
        number of positions it has cached) -> logits of the last position
        (vocab,), or of every position (seq_len, vocab) (executor.py:282-341)."""
        if seq_id not in self._slot:
            raise ValueError(f"unknown sequence {seq_id}")
        ids = [int(t) for t in np.asarray(token_ids).reshape(-1)]
        self._check_tokens(ids)
        if start_position != self._len[seq_id]:
            raise ValueError(f"sequence {seq_id} holds {self._len[seq_id]} positions; start_position "
                             f"{start_position} must continue it (truncate_sequence rewinds)")
        if start_position + len(ids) > self.capacity:
            raise ValueError(f"sequence {seq_id} would exceed the cache capacity of {self.capacity} positions")
        slot = self._slot[seq_id]
        chunks = []
        with torch.cuda.device(self.device):
            for c0 in range(0, len(ids), _ROWS):
                part = ids[c0:c0 + _ROWS]
                pos = [start_position + c0 + j for j in range(len(part))]
                logits = self._forward([slot] * len(part), part, pos)
                chunks.append(logits.clone() if return_all_positions else logits[-1:].clone())
            out = torch.cat(chunks).cpu().numpy()
        self._len[seq_id] = start_position + len(ids)
        return out if return_all_positions else out[-1]

    def forward_batch_decode(self, seq_ids: Sequence[int], token_ids: Sequence[int],
                             positions: Sequence[int]) -> np.ndarray:
        """One decode token for each of N sequences at once -> logits (N, vocab)
        (executor.py:343-396)."""
        n = len(seq_ids)
        if not (len(token_ids) == len(positions) == n):
            raise ValueError("seq_ids, token_ids, and positions must be the same length.")
        if len(set(seq_ids)) != n:
            raise ValueError("forward_batch_decode takes each sequence once")
        for s, p in zip(seq_ids, positions):
            if s not in self._slot:
                raise ValueError(f"unknown sequence {s}")
            if int(p) != self._len[s] or int(p) >= self.capacity:
                raise ValueError(f"sequence {s}: position {p} must continue its {self._len[s]} cached positions "
                                 f"within the capacity of {self.capacity}")
        ids = [int(t) for t in token_ids]
        self._check_tokens(ids)
        outs = []
        with torch.cuda.device(self.device):
            for c0 in range(0, n, _ROWS):
                sl = slice(c0, c0 + _ROWS)
                outs.append(self._forward([self._slot[s] for s in seq_ids[sl]], ids[sl],
                                          [int(p) for p in positions[sl]]).clone())
            out = torch.cat(outs).cpu().numpy()
        for s in seq_ids:
            self._len[s] += 1
        return out

    def generate_greedy(self, prompt_ids: Sequence[int], max_new_tokens: int) -> List[int]:
        """Greedy generation (executor.py:398-413)."""
        seq_id = self.new_sequence()
        try:
            ids = list(prompt_ids)
            logits = self.forward_step(seq_id, np.array(ids), 0)
            for _ in range(max_new_tokens):
                nxt = int(np.argmax(logits))
                ids.append(nxt)
                logits = self.forward_step(seq_id, np.array([nxt]), len(ids) - 1)
            return ids
        finally:
            self.end_sequence(seq_id)
