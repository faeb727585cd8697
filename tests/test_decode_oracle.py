"""The decode-step oracle (oracle/llama_decode.py) is pinned to the reference
executor's own logits on three fixtures (tests/golden/make_decode_golden.py
ran draco.runtime.cpu.executor on each): tiny_llama_decode.gguf (every GPU
block type), tiny_qwen2_decode.gguf (q/k/v and o_proj biases, tied
embeddings, rope base 1e6) and tiny_fused_decode.gguf (a fused q/k/v weight
with grouped-query rows, gate/up/down biases)."""

from pathlib import Path

import numpy as np
import pytest

from dracort_b200.format.gguf_file import GGUFFile
from oracle import llama_decode as D
from oracle.llama_decode import OracleLlama

HERE = Path(__file__).resolve().parent / "golden"


FIXTURES = ["tiny_llama_decode", "tiny_qwen2_decode", "tiny_fused_decode"]


@pytest.fixture(scope="module", params=FIXTURES)
def name(request):
    return request.param


@pytest.fixture(scope="module")
def ref(name):
    return np.load(HERE / f"{name}_ref.npz")


@pytest.fixture()
def model(name):
    gf = GGUFFile(str(HERE / f"{name}.gguf"))
    try:
        yield OracleLlama(gf, q6k_order="d_first")
    finally:
        gf.close()


def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_oracle_prefill_matches_reference_executor(model, ref):
    s = model.new_sequence()
    got = model.forward_step(s, ref["prompt"], 0, return_all_positions=True)
    assert got.shape == ref["prefill_logits"].shape
    assert rel(got, ref["prefill_logits"]) < 1e-6


def test_oracle_greedy_decode_matches_reference_executor(model, ref):
    s = model.new_sequence()
    ids = list(ref["prompt"])
    logits = model.forward_step(s, np.array(ids), 0)
    for t_ref, l_ref in zip(ref["decode_tokens"], ref["decode_logits"]):
        t = int(np.argmax(logits))
        assert t == int(t_ref)
        ids.append(t)
        logits = model.forward_step(s, np.array([t]), len(ids) - 1)
        assert rel(logits, l_ref) < 1e-6


def test_oracle_batch_decode_matches_reference_executor(model, ref):
    sa, sb = model.new_sequence(), model.new_sequence()
    la = model.forward_step(sa, ref["prompt"], 0)
    lb = model.forward_step(sb, ref["prompt_b"], 0)
    toks = [int(np.argmax(la)), int(np.argmax(lb))]
    assert toks == [int(t) for t in ref["batch_tokens"]]
    got = model.forward_batch_decode([sa, sb], toks, [len(ref["prompt"]), len(ref["prompt_b"])])
    assert rel(got, ref["batch_logits"]) < 1e-6


def test_product_rope_tables_equal_the_reference_construction():
    from dracort_b200.gguf_executor import LlamaConfig, rope_tables
    from oracle.llama_decode import build_rope_cache

    gf = GGUFFile(str(HERE / "tiny_llama_decode.gguf"))
    try:
        cfg = LlamaConfig.from_gguf(gf)
    finally:
        gf.close()
    assert (cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.vocab_size) == (256, 8, 4, 96)
    assert not cfg.tie_word_embeddings and cfg.head_dim == 32
    c, s = rope_tables(cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta)
    rc, rs = build_rope_cache(cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta)
    assert np.array_equal(c.view(np.uint32), rc.astype(np.float32).view(np.uint32))
    assert np.array_equal(s.view(np.uint32), rs.astype(np.float32).view(np.uint32))


def test_layer_decode_step_equals_the_oracle_model():
    """layer_decode_step + head_step over array caches reproduce
    OracleLlama.forward_step for a decode token (the form the decode-step
    benchmark's CPU baseline times)."""
    gf = GGUFFile(str(HERE / "tiny_llama_decode.gguf"))
    try:
        m = D.OracleLlama(gf, "d_first")
    finally:
        gf.close()
    cfg = m.cfg
    heads, kvh, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], m.head_dim
    s = m.new_sequence()
    prompt = [1, 5, 17, 42, 7, 63]
    m.forward_step(s, prompt, 0)
    pos, tok = len(prompt), 9
    caches = []
    for layer in range(cfg["num_hidden_layers"]):
        kc = np.zeros((16, kvh, hd), dtype=np.float32)
        vc = np.zeros_like(kc)
        kc[:pos] = np.stack(m.kv[s][layer][0])
        vc[:pos] = np.stack(m.kv[s][layer][1])
        caches.append((kc, vc))
    want = m.forward_step(s, [tok], pos)
    hidden = m.w["token_embd.weight"][[tok]].astype(np.float32)
    for layer, (kc, vc) in enumerate(caches):
        p = f"blk.{layer}."
        w = {"attn_norm": m.w[p + "attn_norm.weight"], "q": m.w[p + "attn_q.weight"], "k": m.w[p + "attn_k.weight"],
             "v": m.w[p + "attn_v.weight"], "o": m.w[p + "attn_output.weight"],
             "ffn_norm": m.w[p + "ffn_norm.weight"], "gate": m.w[p + "ffn_gate.weight"],
             "up": m.w[p + "ffn_up.weight"], "down": m.w[p + "ffn_down.weight"]}
        hidden = D.layer_decode_step(hidden, w, kc, vc, pos, m.cos, m.sin, cfg["rms_norm_eps"], heads, kvh)
    got = D.head_step(hidden, m.w["output_norm.weight"], m.w["output.weight"], cfg["rms_norm_eps"])[0]
    assert np.allclose(got, want, rtol=1e-6, atol=1e-6)


def test_layer_decode_batch_equals_the_oracle_model():
    """layer_decode_batch + head_step reproduce OracleLlama.forward_batch_decode
    for two sequences at different lengths."""
    gf = GGUFFile(str(HERE / "tiny_llama_decode.gguf"))
    try:
        m = D.OracleLlama(gf, "d_first")
    finally:
        gf.close()
    cfg = m.cfg
    heads, kvh, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], m.head_dim
    prompts = [[1, 5, 17, 42, 7, 63], [3, 88, 12]]
    seqs = [m.new_sequence() for _ in prompts]
    for sq, pr in zip(seqs, prompts):
        m.forward_step(sq, pr, 0)
    toks, lengths = [11, 30], [len(p) for p in prompts]
    caches = []
    for layer in range(cfg["num_hidden_layers"]):
        per = []
        for sq, n0 in zip(seqs, lengths):
            kc = np.zeros((16, kvh, hd), dtype=np.float32)
            vc = np.zeros_like(kc)
            kc[:n0] = np.stack(m.kv[sq][layer][0])
            vc[:n0] = np.stack(m.kv[sq][layer][1])
            per.append((kc, vc))
        caches.append(per)
    want = m.forward_batch_decode(seqs, toks, lengths)
    hidden = m.w["token_embd.weight"][toks].astype(np.float32)
    for layer in range(cfg["num_hidden_layers"]):
        p = f"blk.{layer}."
        w = {"attn_norm": m.w[p + "attn_norm.weight"], "q": m.w[p + "attn_q.weight"], "k": m.w[p + "attn_k.weight"],
             "v": m.w[p + "attn_v.weight"], "o": m.w[p + "attn_output.weight"],
             "ffn_norm": m.w[p + "ffn_norm.weight"], "gate": m.w[p + "ffn_gate.weight"],
             "up": m.w[p + "ffn_up.weight"], "down": m.w[p + "ffn_down.weight"]}
        hidden = D.layer_decode_batch(hidden, w, caches[layer], lengths, m.cos, m.sin, cfg["rms_norm_eps"], heads, kvh)
    got = D.head_step(hidden, m.w["output_norm.weight"], m.w["output.weight"], cfg["rms_norm_eps"])
    assert np.allclose(got, want, rtol=1e-6, atol=1e-6)


def test_fixture_flags_follow_the_reference_mapping():
    """gguf.py:765-768: the flags come from layer 0's tensors."""
    want = {"tiny_llama_decode": (False, False, False, False),
            "tiny_qwen2_decode": (False, True, False, True),
            "tiny_fused_decode": (True, False, True, False)}
    for nm, flags in want.items():
        gf = GGUFFile(str(HERE / f"{nm}.gguf"))
        try:
            cfg = D.config_from_metadata(gf.metadata, gf.tensors)
        finally:
            gf.close()
        assert (cfg["qkv_fused"], cfg["attention_bias"], cfg["mlp_bias"], cfg["tie_word_embeddings"]) == flags, nm
