"""Generate the GGUF-container fixtures in tests/golden/ and pin them with the
REAL reference reader.

    python tests/golden/make_gguf_golden.py --reference /path/to/DracoRT

1. ``tiny_llama.gguf``: a small llama-architecture GGUF v3 file (one decoder
   layer, hidden 256, ffn 512) written by dracort_b200.format.gguf_file.write_gguf
   with seeded N(0, 0.02) weights: Q4_K q/gate/down, Q8_0 k, Q6_K v (in the
   d-first byte order the reference decodes), F32 norms, an F16 embedding, and
   metadata of every value type including string and float arrays.
2. ``tiny_llama_ref.npz``: what the reference's own GGUFReader
   (draco/format/gguf.py:528-662) reports for that file — per tensor the
   canonical name, ggml type, shape, absolute offset and byte count — and the
   SHA-256 of the fp32 array its get_tensor (gguf.py:820-834) returns, plus
   a few of its values and the parsed metadata it exposes.

Nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from dracort_b200.format import quantize as Q  # noqa: E402
from dracort_b200.format.gguf_file import write_gguf  # noqa: E402

HIDDEN, FFN, VOCAB = 256, 512, 64


def build(path: Path) -> None:
    rng = np.random.default_rng(4242)
    w = lambda n, k: Q.random_weight(rng, n, k)  # noqa: E731
    tensors = [
        ("token_embd.weight", 1, (VOCAB, HIDDEN), (rng.standard_normal((VOCAB, HIDDEN)) * 0.02).astype(np.float16).tobytes()),
        ("blk.0.attn_norm.weight", 0, (HIDDEN,), (1 + 0.1 * rng.standard_normal(HIDDEN)).astype(np.float32).tobytes()),
        ("blk.0.attn_q.weight", 12, (HIDDEN, HIDDEN), Q.encode(12, w(HIDDEN, HIDDEN)).tobytes()),
        ("blk.0.attn_k.weight", 8, (HIDDEN, HIDDEN), Q.encode(8, w(HIDDEN, HIDDEN)).tobytes()),
        ("blk.0.attn_v.weight", 14, (HIDDEN, HIDDEN), Q.encode(14, w(HIDDEN, HIDDEN)).tobytes()),
        ("blk.0.attn_output.weight", 12, (HIDDEN, HIDDEN), Q.encode(12, w(HIDDEN, HIDDEN)).tobytes()),
        ("blk.0.ffn_norm.weight", 0, (HIDDEN,), (1 + 0.1 * rng.standard_normal(HIDDEN)).astype(np.float32).tobytes()),
        ("blk.0.ffn_gate.weight", 12, (FFN, HIDDEN), Q.encode(12, w(FFN, HIDDEN)).tobytes()),
        ("blk.0.ffn_up.weight", 8, (FFN, HIDDEN), Q.encode(8, w(FFN, HIDDEN)).tobytes()),
        ("blk.0.ffn_down.weight", 12, (HIDDEN, FFN), Q.encode(12, w(HIDDEN, FFN)).tobytes()),
        ("output_norm.weight", 0, (HIDDEN,), np.ones(HIDDEN, dtype=np.float32).tobytes()),
    ]
    meta = {
        "general.architecture": "llama",
        "general.name": "tiny-llama-fixture",
        "llama.embedding_length": HIDDEN,
        "llama.block_count": 1,
        "llama.feed_forward_length": FFN,
        "llama.attention.head_count": 8,
        "llama.attention.head_count_kv": 4,
        "llama.context_length": 128,
        "llama.rope.freq_base": 10000.0,
        "llama.attention.layer_norm_rms_epsilon": 1e-5,
        "llama.vocab_size": VOCAB,
        "general.quantized": True,
        "general.file_type": 15,
        "tokenizer.ggml.model": "llama",
        "tokenizer.ggml.tokens": [f"<t{i}>" for i in range(VOCAB)],
        "tokenizer.ggml.scores": [float(-i) for i in range(VOCAB)],
        "tokenizer.ggml.token_type": [1] * VOCAB,
        "tokenizer.ggml.bos_token_id": 1,
        "tokenizer.ggml.eos_token_id": 2,
    }
    write_gguf(str(path), tensors, meta)


def load_reference_reader(ref: Path):
    import types

    d = ref / "draco"
    for name, sub in [("draco", ""), ("draco.format", "format"), ("draco.utils", "utils")]:
        if name not in sys.modules:
            m = types.ModuleType(name)
            m.__path__ = [str(d / sub)]
            sys.modules[name] = m
    import draco.format.gguf as gguf  # noqa: E402

    return gguf


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DRACO_REFERENCE"),
                    help="path of the DracoRT checkout (default: $DRACO_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        raise SystemExit("give the reference checkout: --reference PATH or DRACO_REFERENCE=PATH")
    path = HERE / "tiny_llama.gguf"
    build(path)
    gguf = load_reference_reader(Path(a.reference))
    out = {}
    rows = []
    with gguf.GGUFReader(str(path)) as r:
        for info in r.tensors():
            arr = r.get_tensor(info.name)
            rows.append({"name": info.name, "ggml_type": info.ggml_type, "shape": list(info.shape),
                         "offset": info.offset, "nbytes": info.nbytes,
                         "sha256": hashlib.sha256(np.ascontiguousarray(arr, dtype=np.float32).tobytes()).hexdigest(),
                         "head": [float(v) for v in arr.reshape(-1)[:4]]})
        out["metadata"] = json.dumps(r.metadata, sort_keys=True)
        out["tokens_head"] = json.dumps(r.tokenizer["tokens"][:4]) if r.tokenizer else "[]"
    out["index"] = json.dumps(rows)
    np.savez_compressed(HERE / "tiny_llama_ref.npz", **{k: np.array(v) for k, v in out.items()})
    print(f"wrote {path} ({path.stat().st_size} B) and tiny_llama_ref.npz: {len(rows)} tensors")


if __name__ == "__main__":
    main()
