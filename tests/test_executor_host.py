"""Host logic of GPUExecutionBackend that needs no GPU: the llama configuration
read from GGUF metadata (draco/format/gguf.py:680-770), the key/value cache
sizing from CPUExecutionBackend's arguments (executor.py:133-159), the
constructor's argument checks, and the RoPE tables (build_rope_cache,
draco/runtime/cpu/ops.py:77-83)."""

from pathlib import Path

import numpy as np
import pytest

from dracort_b200.format.gguf_file import GGUFFile
from dracort_b200.gguf_executor import GPUExecutionBackend, LlamaConfig, cache_capacity, rope_tables
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
