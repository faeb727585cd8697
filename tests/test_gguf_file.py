"""The GGUF container reader / writer (dracort_b200.format.gguf_file) on CPU.

Pinned against the reference's own GGUFReader (draco/format/gguf.py:528-662)
through tests/golden/tiny_llama_ref.npz (made by tests/golden/make_gguf_golden.py):
the same tensor index (names, types, shapes, absolute offsets, byte counts),
and payloads whose CPU-oracle decode hashes to what the reference's
get_tensor (gguf.py:820-834) returned.  Plus the reference's error cases
(gguf.py:535-552, 640-644) and a write/read round trip of every metadata type.
"""

import hashlib
import json
import os
import struct

import numpy as np
import pytest

from dracort_b200.exceptions import DracoFormatError
from dracort_b200.format.gguf_file import GGUFFile, canonical_name, tensor_nbytes, write_gguf
from oracle import gguf_oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TINY = os.path.join(GOLDEN, "tiny_llama.gguf")


@pytest.fixture(scope="module")
def ref():
    z = np.load(os.path.join(GOLDEN, "tiny_llama_ref.npz"))
    return {"index": json.loads(str(z["index"])), "metadata": json.loads(str(z["metadata"])),
            "tokens_head": json.loads(str(z["tokens_head"]))}


def _host_decode(gf, t):
    """fp32 array the reference's get_tensor returns, via the CPU oracle."""
    p = gf.payload(t.name)
    if t.ggml_type == 0:
        return p.view(np.float32).reshape(t.shape)
    if t.ggml_type == 1:
        return p.view(np.float16).astype(np.float32).reshape(t.shape)
    return O.dequantize(t.ggml_type, p, t.n_elements).reshape(t.shape)


def test_index_matches_reference_reader(ref):
    with GGUFFile(TINY) as gf:
        mine = {canonical_name(t.name): t for t in gf}
        assert len(mine) == len(ref["index"])
        for row in ref["index"]:
            t = mine[row["name"]]
            assert (t.ggml_type, list(t.shape), t.offset, t.nbytes) == \
                   (row["ggml_type"], row["shape"], row["offset"], row["nbytes"]), row["name"]


def test_payloads_decode_to_the_reference_tensors(ref):
    with GGUFFile(TINY) as gf:
        mine = {canonical_name(t.name): t for t in gf}
        for row in ref["index"]:
            arr = np.ascontiguousarray(_host_decode(gf, mine[row["name"]]), dtype=np.float32)
            assert hashlib.sha256(arr.tobytes()).hexdigest() == row["sha256"], row["name"]


def test_metadata(ref):
    with GGUFFile(TINY) as gf:
        md = gf.metadata
        assert gf.version == 3 and gf.architecture == "llama" and gf.alignment == 32
        assert md["llama.embedding_length"] == ref["metadata"]["hidden_size"] == 256
        assert md["llama.block_count"] == ref["metadata"]["num_hidden_layers"]
        assert md["llama.attention.head_count_kv"] == ref["metadata"]["num_key_value_heads"]
        assert md["tokenizer.ggml.tokens"][:4] == ref["tokens_head"]
        assert md["tokenizer.ggml.scores"][:3] == [0.0, -1.0, -2.0]
        assert md["general.quantized"] is True
        assert gf.data_offset % 32 == 0


def test_canonical_names():
    assert canonical_name("blk.3.attn_q.weight") == "model.layers.3.self_attn.q_proj.weight"
    assert canonical_name("blk.0.ffn_down.weight") == "model.layers.0.mlp.down_proj.weight"
    assert canonical_name("token_embd.weight") == "model.embed_tokens.weight"
    assert canonical_name("blk.1.attn_q.bias") == "model.layers.1.self_attn.q_proj.bias"
    assert canonical_name("something.else") == "something.else"


def test_round_trip_every_value_type(tmp_path):
    rng = np.random.default_rng(3)
    q = O.BLOCK_LAYOUTS
    from dracort_b200.format import quantize as Q

    w = Q.encode(12, Q.random_weight(rng, 32, 512))
    f = (rng.standard_normal((3, 5))).astype(np.float32)
    meta = {"u32": 7, "u64": 2 ** 40, "i64": -5, "f": 0.5, "b": False, "s": "naïve",
            "arr_i": [1, 2, 3], "arr_neg": [-1, 2], "arr_s": ["a", "bc"], "arr_f": [0.25, 1.5], "arr_b": [True, False]}
    p = tmp_path / "rt.gguf"
    write_gguf(str(p), [("w", 12, (32, 512), w.tobytes()), ("f", 0, (3, 5), f.tobytes())], meta, alignment=64)
    with GGUFFile(str(p)) as gf:
        for k, v in meta.items():
            assert gf.metadata[k] == v, k
        assert gf.alignment == 64 and gf.data_offset % 64 == 0
        t = gf.tensor("w")
        assert (t.n_rows, t.k, t.nbytes, t.offset % 64) == (32, 512, w.nbytes, 0)
        assert np.array_equal(gf.payload("w").reshape(w.shape), w)
        assert np.array_equal(gf.payload("f").view(np.float32).reshape(3, 5), f)
        with pytest.raises(KeyError):
            gf.tensor("missing")
    assert q[12] == (256, 144)


def _header(version=3, n_t=0, n_kv=0, magic=b"GGUF"):
    return magic + struct.pack("<IQQ", version, n_t, n_kv)


def test_errors_like_the_reference(tmp_path):
    cases = {
        "magic": _header(magic=b"GGML") + b"\0" * 8,
        "version": _header(version=4) + b"\0" * 8,
        "small": b"GGUF\x03",
        "truncated": _header(n_kv=1) + struct.pack("<Q", 100) + b"abc",
        "alignment": _header(n_kv=1) + struct.pack("<Q", 17) + b"general.alignment" + struct.pack("<II", 4, 12),
    }
    for name, blob in cases.items():
        p = tmp_path / f"{name}.gguf"
        p.write_bytes(blob)
        with pytest.raises(DracoFormatError):
            GGUFFile(str(p))
    # a tensor that runs past the end of the file
    p = tmp_path / "short.gguf"
    write_gguf(str(p), [("f", 0, (64,), np.zeros(64, np.float32).tobytes())])
    p.write_bytes(p.read_bytes()[:-8])
    with pytest.raises(DracoFormatError, match="past the end"):
        GGUFFile(str(p))
    # quantized rows must hold whole blocks (gguf.py:640-644)
    with pytest.raises(DracoFormatError):
        tensor_nbytes(12, (4, 100))


def test_shard_ranges():
    from dracort_b200.format.gguf_file import GGUFTensor
    from dracort_b200.gguf_loader import Shard, _shard_ranges

    t = GGUFTensor("w", 12, (4096, 11008), 0, tensor_nbytes(12, (4096, 11008)))
    ks = [_shard_ranges(t, Shard("row", r, 8))[2:] for r in range(8)]
    assert [(b - a) // 256 for a, b in ks] == [6, 6, 6, 5, 5, 5, 5, 5] and ks[-1][1] == 11008
    rs = [_shard_ranges(t, Shard("col", r, 4))[:2] for r in range(4)]
    assert rs == [(0, 1024), (1024, 2048), (2048, 3072), (3072, 4096)]
    with pytest.raises(ValueError):
        Shard("diag", 0, 2)
