"""Host logic of GPUExecutionBackend that needs no GPU: the llama configuration
read from GGUF metadata (draco/format/gguf.py:680-770) and the tensors each
layer takes under its flags (biases, a fused q/k/v weight), the key/value cache
sizing from CPUExecutionBackend's arguments (executor.py:133-159), the
constructor's argument checks, and the RoPE tables (build_rope_cache,
draco/runtime/cpu/ops.py:77-83)."""

from pathlib import Path

import numpy as np
import pytest

from dracort_b200.format.gguf_file import GGUFFile
from dracort_b200.format.gguf_types import BLOCK_LAYOUTS
from dracort_b200.gguf_executor import GPUExecutionBackend, LlamaConfig, cache_capacity, layer_tensors, rope_tables
from oracle import gguf_oracle as O
from oracle import llama_decode as D

FIXTURE = Path(__file__).resolve().parent / "golden" / "tiny_llama_decode.gguf"


@pytest.fixture(scope="module")
def cfg():
    gf = GGUFFile(str(FIXTURE))
    try:
        return LlamaConfig.from_gguf(gf)
    finally:
        gf.close()


def test_config_matches_the_oracle_mapping(cfg):
    gf = GGUFFile(str(FIXTURE))
    try:
        ref = D.config_from_metadata(gf.metadata, gf.tensors)
    finally:
        gf.close()
    assert cfg.hidden_size == ref["hidden_size"] == 256
    assert cfg.num_hidden_layers == ref["num_hidden_layers"] == 2
    assert cfg.num_attention_heads == ref["num_attention_heads"] == 8
    assert cfg.num_key_value_heads == ref["num_key_value_heads"] == 4
    assert cfg.max_position_embeddings == ref["max_position_embeddings"] == 64
    assert cfg.rope_theta == ref["rope_theta"]
    assert np.float32(cfg.rms_norm_eps) == np.float32(ref["rms_norm_eps"])
    assert cfg.head_dim == 32


def test_cache_capacity_from_the_reference_arguments(cfg):
    # per position, two sequences: 2 seqs x 2 layers x (k, v) x 4 heads x 32 x 4 B
    per_pos = 2 * 2 * 2 * 4 * 32 * 4
    assert cache_capacity(cfg, 2) == 64  # the context length
    assert cache_capacity(cfg, 2, max_seq_len=10) == 10
    assert cache_capacity(cfg, 2, max_seq_len=1000) == 64  # never above the context
    assert cache_capacity(cfg, 2, kv_budget_bytes=24 * per_pos + 5) == 24
    assert cache_capacity(cfg, 2, kv_budget_bytes=1 << 40) == 64
    assert cache_capacity(cfg, 2, max_seq_len=8, kv_budget_bytes=1) == 8  # max_seq_len wins
    with pytest.raises(ValueError, match="holds no position"):
        cache_capacity(cfg, 2, kv_budget_bytes=per_pos - 1)


def test_constructor_argument_checks():
    with pytest.raises(ValueError, match="CUDA device"):
        GPUExecutionBackend(str(FIXTURE), device="cpu")
    with pytest.raises(ValueError, match="fp32 cache"):
        GPUExecutionBackend(str(FIXTURE), 1, "f16")
    with pytest.raises(TypeError, match="path"):
        GPUExecutionBackend(object())


def test_rope_tables_are_the_reference_formula():
    cos, sin = rope_tables(32, 64, 10000.0)
    ocos, osin = D.build_rope_cache(32, 64, 10000.0)
    assert cos.dtype == np.float32 and cos.shape == (64, 16)
    assert np.array_equal(cos, ocos.astype(np.float32)) and np.array_equal(sin, osin.astype(np.float32))


def _cfg_and_names(name):
    gf = GGUFFile(str(FIXTURE.parent / f"{name}.gguf"))
    try:
        return LlamaConfig.from_gguf(gf), list(gf.tensors)
    finally:
        gf.close()


def test_layer_tensors_plain_llama():
    cfg, names = _cfg_and_names("tiny_llama_decode")
    assert (cfg.qkv_fused, cfg.attention_bias, cfg.mlp_bias, cfg.tie_word_embeddings) == (False, False, False, False)
    t = layer_tensors(cfg, names, 1)
    assert t["proj"]["q"] == ("blk.1.attn_q.weight", None)
    assert t["proj"]["down"] == ("blk.1.ffn_down.weight", None)
    assert all(b is None for b in t["bias"].values())
    assert (t["attn_norm"], t["ffn_norm"]) == ("blk.1.attn_norm.weight", "blk.1.ffn_norm.weight")


def test_layer_tensors_qwen2_biases():
    cfg, names = _cfg_and_names("tiny_qwen2_decode")
    assert (cfg.qkv_fused, cfg.attention_bias, cfg.mlp_bias, cfg.tie_word_embeddings) == (False, True, False, True)
    assert cfg.rope_theta == 1e6
    t = layer_tensors(cfg, names, 0)
    assert t["bias"] == {"q": "blk.0.attn_q.bias", "k": "blk.0.attn_k.bias", "v": "blk.0.attn_v.bias",
                         "o": "blk.0.attn_output.bias", "gate": None, "up": None, "down": None}


def test_layer_tensors_fused_qkv_rows_and_mlp_biases():
    cfg, names = _cfg_and_names("tiny_fused_decode")
    assert (cfg.qkv_fused, cfg.attention_bias, cfg.mlp_bias) == (True, False, True)
    t = layer_tensors(cfg, names, 1)
    fused = "blk.1.attn_qkv.weight"
    # 8 query heads and 4 key/value heads of 32: q rows 0-255, k 256-383, v 384-511
    assert (t["proj"]["q"], t["proj"]["k"], t["proj"]["v"]) == ((fused, (0, 256)), (fused, (256, 384)),
                                                                (fused, (384, 512)))
    assert t["proj"]["o"] == ("blk.1.attn_output.weight", None)
    assert t["bias"] == {"q": None, "k": None, "v": None, "o": None, "gate": "blk.1.ffn_gate.bias",
                         "up": "blk.1.ffn_up.bias", "down": "blk.1.ffn_down.bias"}


def test_fused_row_ranges_dequantize_to_the_fused_rows():
    """Rows of a packed GGUF weight are independent: the q/k/v row ranges the
    executor regroups decode to the fused weight's rows."""
    gf = GGUFFile(str(FIXTURE.parent / "tiny_fused_decode.gguf"))
    try:
        for layer in (0, 1):
            t = gf.tensor(f"blk.{layer}.attn_qkv.weight")
            bs, bb = BLOCK_LAYOUTS[t.ggml_type]
            rows = np.asarray(gf.payload(t.name)).reshape(t.n_rows, t.k // bs * bb)
            full = O.dequantize_matrix(t.ggml_type, rows, t.n_rows, t.k)
            for r0, r1 in ((0, 256), (256, 384), (384, 512)):
                part = O.dequantize_matrix(t.ggml_type, np.ascontiguousarray(rows[r0:r1]), r1 - r0, t.k)
                assert np.array_equal(part, full[r0:r1])
    finally:
        gf.close()
