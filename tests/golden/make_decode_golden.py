"""Generate the decode-step fixtures in tests/golden/ and pin them with the
REAL reference executor.

    python tests/golden/make_decode_golden.py --reference /path/to/DracoRT

1. ``tiny_llama_decode.gguf``: a two-layer llama-architecture GGUF v3 file
   (hidden 256, 8 query heads and 4 key/value heads of 32, ffn 512, vocab 96)
   written by dracort_b200.format.gguf_file.write_gguf with seeded weights in
   every GPU block type (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K in the
   d-first byte order the reference decodes), an F16 embedding, F32 norms and
   a Q6_K output head.
2. ``tiny_qwen2_decode.gguf``: the same shapes as a qwen2 file — q/k/v and
   o_proj biases (F32) in every layer, tied embeddings (no output tensor),
   rope base 1e6 — and ``tiny_fused_decode.gguf``: a llama file with one fused
   q/k/v weight per layer (``attn_qkv``, grouped-query rows) and gate/up/down
   biases;
3. ``<name>_ref.npz`` for each file: what the reference's own CPU executor
   (draco/runtime/cpu/executor.py: CPUExecutionBackend over
   draco/format/gguf.py: GGUFReader) computes on it:
     * ``prefill_logits`` — forward_step over a 6-token prompt with
       return_all_positions (executor.py:282-341): the logits of every position;
     * ``decode_tokens`` / ``decode_logits`` — greedy steps after that prompt,
       each a forward_step of one token (the loop of engine/llm.py:1158-1199);
     * ``batch_logits`` — forward_batch_decode (executor.py:343-396) of two
       sequences with different prompt lengths, one token each.

Nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from dracort_b200.format import quantize as Q  # noqa: E402
from dracort_b200.format.gguf_file import write_gguf  # noqa: E402

HIDDEN, FFN, VOCAB, HEADS, KV_HEADS = 256, 512, 96, 8, 4
HEAD_DIM = HIDDEN // HEADS
PROMPT = [1, 5, 17, 42, 7, 63]
PROMPT_B = [3, 88, 12]
DECODE_STEPS = 4

# per layer: (q, k, v, o, gate, up, down) ggml types
LAYER_TYPES = [
    (12, 8, 14, 12, 12, 13, 12),  # Q4_K, Q8_0, Q6_K, Q4_K, Q4_K, Q5_K, Q4_K
    (2, 3, 7, 8, 14, 6, 13),      # Q4_0, Q4_1, Q5_1, Q8_0, Q6_K, Q5_0, Q5_K
]


def build(path: Path) -> None:
    rng = np.random.default_rng(9090)

    def quant(qt, n, k, std=0.05):
        return Q.encode(qt, Q.random_weight(rng, n, k, std=std)).tobytes()  # Q6_K in the d-first order

    def norm_w(n):
        return (1 + 0.1 * rng.standard_normal(n)).astype(np.float32).tobytes()

    kv = KV_HEADS * HEAD_DIM
    tensors = [("token_embd.weight", 1, (VOCAB, HIDDEN),
                (rng.standard_normal((VOCAB, HIDDEN)) * 0.5).astype(np.float16).tobytes())]
    for layer, (tq, tk, tv, to, tg, tu, td) in enumerate(LAYER_TYPES):
        p = f"blk.{layer}."
        tensors += [
            (p + "attn_norm.weight", 0, (HIDDEN,), norm_w(HIDDEN)),
            (p + "attn_q.weight", tq, (HIDDEN, HIDDEN), quant(tq, HIDDEN, HIDDEN)),
            (p + "attn_k.weight", tk, (kv, HIDDEN), quant(tk, kv, HIDDEN)),
            (p + "attn_v.weight", tv, (kv, HIDDEN), quant(tv, kv, HIDDEN)),
            (p + "attn_output.weight", to, (HIDDEN, HIDDEN), quant(to, HIDDEN, HIDDEN)),
            (p + "ffn_norm.weight", 0, (HIDDEN,), norm_w(HIDDEN)),
            (p + "ffn_gate.weight", tg, (FFN, HIDDEN), quant(tg, FFN, HIDDEN)),
            (p + "ffn_up.weight", tu, (FFN, HIDDEN), quant(tu, FFN, HIDDEN)),
            (p + "ffn_down.weight", td, (HIDDEN, FFN), quant(td, HIDDEN, FFN)),
        ]
    tensors += [
        ("output_norm.weight", 0, (HIDDEN,), norm_w(HIDDEN)),
        ("output.weight", 14, (VOCAB, HIDDEN), quant(14, VOCAB, HIDDEN)),
    ]
    meta = {
        "general.architecture": "llama",
        "general.name": "tiny-llama-decode-fixture",
        "llama.embedding_length": HIDDEN,
        "llama.block_count": len(LAYER_TYPES),
        "llama.feed_forward_length": FFN,
        "llama.attention.head_count": HEADS,
        "llama.attention.head_count_kv": KV_HEADS,
        "llama.context_length": 64,
        "llama.rope.freq_base": 10000.0,
        "llama.attention.layer_norm_rms_epsilon": 1e-5,
        "llama.vocab_size": VOCAB,
    }
    write_gguf(str(path), tensors, meta)


def _common_meta(arch: str, theta: float = 10000.0) -> dict:
    p = arch + "."
    return {
        "general.architecture": arch,
        "general.name": f"tiny-{arch}-decode-fixture",
        p + "embedding_length": HIDDEN,
        p + "block_count": len(LAYER_TYPES),
        p + "feed_forward_length": FFN,
        p + "attention.head_count": HEADS,
        p + "attention.head_count_kv": KV_HEADS,
        p + "context_length": 64,
        p + "rope.freq_base": theta,
        p + "attention.layer_norm_rms_epsilon": 1e-5,
        p + "vocab_size": VOCAB,
    }


def build_qwen2(path: Path) -> None:
    """qwen2-style: biases on q/k/v and o_proj, tied embeddings, rope base 1e6."""
    rng = np.random.default_rng(9191)

    def quant(qt, n, k, std=0.05):
        return Q.encode(qt, Q.random_weight(rng, n, k, std=std)).tobytes()

    def vec(n, scale, offset=0.0):
        return (offset + scale * rng.standard_normal(n)).astype(np.float32).tobytes()

    kv = KV_HEADS * HEAD_DIM
    tensors = [("token_embd.weight", 1, (VOCAB, HIDDEN),
                (rng.standard_normal((VOCAB, HIDDEN)) * 0.5).astype(np.float16).tobytes())]
    for layer, (tq, tk, tv, to, tg, tu, td) in enumerate(LAYER_TYPES):
        p = f"blk.{layer}."
        tensors += [
            (p + "attn_norm.weight", 0, (HIDDEN,), vec(HIDDEN, 0.1, 1.0)),
            (p + "attn_q.weight", tq, (HIDDEN, HIDDEN), quant(tq, HIDDEN, HIDDEN)),
            (p + "attn_q.bias", 0, (HIDDEN,), vec(HIDDEN, 0.3)),
            (p + "attn_k.weight", tk, (kv, HIDDEN), quant(tk, kv, HIDDEN)),
            (p + "attn_k.bias", 0, (kv,), vec(kv, 0.3)),
            (p + "attn_v.weight", tv, (kv, HIDDEN), quant(tv, kv, HIDDEN)),
            (p + "attn_v.bias", 0, (kv,), vec(kv, 0.3)),
            (p + "attn_output.weight", to, (HIDDEN, HIDDEN), quant(to, HIDDEN, HIDDEN)),
            (p + "attn_output.bias", 0, (HIDDEN,), vec(HIDDEN, 0.1)),
            (p + "ffn_norm.weight", 0, (HIDDEN,), vec(HIDDEN, 0.1, 1.0)),
            (p + "ffn_gate.weight", tg, (FFN, HIDDEN), quant(tg, FFN, HIDDEN)),
            (p + "ffn_up.weight", tu, (FFN, HIDDEN), quant(tu, FFN, HIDDEN)),
            (p + "ffn_down.weight", td, (HIDDEN, FFN), quant(td, HIDDEN, FFN)),
        ]
    tensors.append(("output_norm.weight", 0, (HIDDEN,), vec(HIDDEN, 0.1, 1.0)))
    write_gguf(str(path), tensors, _common_meta("qwen2", theta=1e6))


def build_fused(path: Path) -> None:
    """llama with a fused q/k/v weight (q rows, then k, then v) per layer and
    gate/up/down biases."""
    rng = np.random.default_rng(9293)

    def quant(qt, n, k, std=0.05):
        return Q.encode(qt, Q.random_weight(rng, n, k, std=std)).tobytes()

    def vec(n, scale, offset=0.0):
        return (offset + scale * rng.standard_normal(n)).astype(np.float32).tobytes()

    qkv_rows = HIDDEN + 2 * KV_HEADS * HEAD_DIM
    fused_types = [12, 8]  # Q4_K, Q8_0
    tensors = [("token_embd.weight", 1, (VOCAB, HIDDEN),
                (rng.standard_normal((VOCAB, HIDDEN)) * 0.5).astype(np.float16).tobytes())]
    for layer, (tq, tk, tv, to, tg, tu, td) in enumerate(LAYER_TYPES):
        p = f"blk.{layer}."
        tf = fused_types[layer]
        tensors += [
            (p + "attn_norm.weight", 0, (HIDDEN,), vec(HIDDEN, 0.1, 1.0)),
            (p + "attn_qkv.weight", tf, (qkv_rows, HIDDEN), quant(tf, qkv_rows, HIDDEN)),
            (p + "attn_output.weight", to, (HIDDEN, HIDDEN), quant(to, HIDDEN, HIDDEN)),
            (p + "ffn_norm.weight", 0, (HIDDEN,), vec(HIDDEN, 0.1, 1.0)),
            (p + "ffn_gate.weight", tg, (FFN, HIDDEN), quant(tg, FFN, HIDDEN)),
            (p + "ffn_gate.bias", 0, (FFN,), vec(FFN, 0.2)),
            (p + "ffn_up.weight", tu, (FFN, HIDDEN), quant(tu, FFN, HIDDEN)),
            (p + "ffn_up.bias", 0, (FFN,), vec(FFN, 0.2)),
            (p + "ffn_down.weight", td, (HIDDEN, FFN), quant(td, HIDDEN, FFN)),
            (p + "ffn_down.bias", 0, (HIDDEN,), vec(HIDDEN, 0.1)),
        ]
    tensors += [
        ("output_norm.weight", 0, (HIDDEN,), vec(HIDDEN, 0.1, 1.0)),
        ("output.weight", 8, (VOCAB, HIDDEN), quant(8, VOCAB, HIDDEN)),
    ]
    write_gguf(str(path), tensors, _common_meta("llama"))


FIXTURES = [("tiny_llama_decode", build), ("tiny_qwen2_decode", build_qwen2), ("tiny_fused_decode", build_fused)]


def load_reference(ref: Path):
    """Import the reference's GGUF reader and CPU executor the way its own
    tests do (tests/conftest.py stubs the top-level packages, so that
    draco/__init__.py, which pulls in the server stack, is not executed)."""
    d = ref / "draco"
    for name, sub in [("draco", ""), ("draco.format", "format"), ("draco.utils", "utils"),
                      ("draco.runtime", "runtime"), ("draco.runtime.cpu", "runtime/cpu"),
                      ("draco.runtime.cpu.kernels", "runtime/cpu/kernels"),
                      ("draco.quantization", "quantization")]:
        if name not in sys.modules:
            m = types.ModuleType(name)
            m.__path__ = [str(d / sub)]
            sys.modules[name] = m
    import draco.format.gguf as gguf  # noqa: E402
    from draco.runtime.cpu.executor import CPUExecutionBackend  # noqa: E402

    return gguf, CPUExecutionBackend


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DRACO_REFERENCE"),
                    help="path of the DracoRT checkout (default: $DRACO_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        raise SystemExit("give the reference checkout: --reference PATH or DRACO_REFERENCE=PATH")
    gguf, Executor = load_reference(Path(a.reference))
    for name, builder in FIXTURES:
        path = HERE / f"{name}.gguf"
        builder(path)
        run_reference(gguf, Executor, path, HERE / f"{name}_ref.npz")


def run_reference(gguf, Executor, path: Path, out_path: Path) -> None:
    out = {"prompt": np.array(PROMPT), "prompt_b": np.array(PROMPT_B)}
    reader = gguf.GGUFReader(str(path))
    ex = Executor(reader, max_num_seqs=2, kv_budget_bytes=64 << 20)
    # every position of the prompt (causal prefill)
    s = ex.new_sequence()
    out["prefill_logits"] = ex.forward_step(s, np.array(PROMPT, dtype=np.int64), 0,
                                            return_all_positions=True).astype(np.float32)
    ex.end_sequence(s)
    # the generation loop: prompt, then one token per step (greedy)
    s = ex.new_sequence()
    ids = list(PROMPT)
    logits = ex.forward_step(s, np.array(ids, dtype=np.int64), 0)
    toks, steps = [], []
    for _ in range(DECODE_STEPS):
        t = int(np.argmax(logits))
        toks.append(t)
        ids.append(t)
        logits = ex.forward_step(s, np.array([t], dtype=np.int64), len(ids) - 1)
        steps.append(np.asarray(logits, dtype=np.float32))
    ex.end_sequence(s)
    out["decode_tokens"] = np.array(toks)
    out["decode_logits"] = np.stack(steps)
    # two sequences decoded together
    sa, sb = ex.new_sequence(), ex.new_sequence()
    la = ex.forward_step(sa, np.array(PROMPT, dtype=np.int64), 0)
    lb = ex.forward_step(sb, np.array(PROMPT_B, dtype=np.int64), 0)
    ta, tb = int(np.argmax(la)), int(np.argmax(lb))
    out["batch_tokens"] = np.array([ta, tb])
    out["batch_logits"] = ex.forward_batch_decode([sa, sb], [ta, tb], [len(PROMPT), len(PROMPT_B)]).astype(np.float32)
    np.savez_compressed(out_path, **out)
    print(f"wrote {path} ({path.stat().st_size} B) and {out_path.name}; decode tokens {toks}, "
          f"batch tokens {[ta, tb]}")


if __name__ == "__main__":
    main()
