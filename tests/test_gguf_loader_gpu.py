"""GGUF file -> GPU (dracort_b200.gguf_loader) against the reference.

The tiny llama file in tests/golden is loaded onto the GPU (pinned staging,
on-device regroup to the TILED layout); dequantizing each loaded weight on
the GPU must hash to the fp32 array the reference's own
GGUFReader.get_tensor (draco/format/gguf.py:820-834) returned for it
(tests/golden/tiny_llama_ref.npz) — bit-exact.  Tensor-parallel shards must
equal slices of the full weight, the Q6_K byte order of llama.cpp files
(d last) must decode like the oracle's d_last order, and a model whose
nn.Linear layers are replaced through GGUFBackend.load_quantized_weights
must match the oracle's linear layers.
"""

import hashlib
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from dracort_b200 import gguf_ops as G  # noqa: E402
from dracort_b200.exceptions import DracoFormatError  # noqa: E402
from dracort_b200.format.gguf_file import GGUFFile, canonical_name, write_gguf  # noqa: E402
from dracort_b200.gguf_loader import DeviceWeight, Shard, load_gguf  # noqa: E402
from oracle import gguf_oracle as O  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TINY = os.path.join(GOLDEN, "tiny_llama.gguf")


def _ref_rows():
    z = np.load(os.path.join(GOLDEN, "tiny_llama_ref.npz"))
    return {r["name"]: r for r in json.loads(str(z["index"]))}


def _sha(t):
    return hashlib.sha256(np.ascontiguousarray(t.float().cpu().numpy(), dtype=np.float32).tobytes()).hexdigest()


def test_loaded_weights_dequantize_to_the_reference_tensors():
    rows = _ref_rows()
    out = load_gguf(TINY, "cuda", q6k_order="d_first", chunk_bytes=1 << 16)  # many staging chunks
    assert len(out) == len(rows)
    for name, v in out.items():
        want = rows[canonical_name(name)]["sha256"]
        if isinstance(v, DeviceWeight):
            deq = G.dequantize(v.qtype, v.tiled, v.n_rows, v.k, layout="tiled")
            assert _sha(deq) == want, name
        else:
            assert _sha(v) == want, name


@pytest.mark.parametrize("kind,world", [("col", 2), ("col", 4), ("row", 2)])
def test_shards_are_slices_of_the_full_weight(kind, world):
    # row shards split k (256-element super-blocks): only ffn_down has two
    names = ["blk.0.ffn_down.weight"] if kind == "row" else [
        "blk.0.ffn_gate.weight", "blk.0.ffn_down.weight", "blk.0.attn_k.weight", "blk.0.attn_v.weight"]
    full = load_gguf(TINY, "cuda", names=names, q6k_order="d_first")
    for r in range(world):
        part = load_gguf(TINY, "cuda", names=names, q6k_order="d_first",
                         shards={n: Shard(kind, r, world) for n in names})
        for n in names:
            f, p = full[n], part[n]
            fd = G.dequantize(f.qtype, f.tiled, f.n_rows, f.k, layout="tiled")
            pd = G.dequantize(p.qtype, p.tiled, p.n_rows, p.k, layout="tiled")
            assert torch.equal(pd, fd[p.r0:p.r1, p.k0:p.k1]), (n, kind, r)
    with pytest.raises(DracoFormatError, match="no super-block"):
        load_gguf(TINY, "cuda", names=["blk.0.attn_k.weight"], shards={"blk.0.attn_k.weight": Shard("row", 1, 2)})


def test_q6k_d_last_files(tmp_path):
    from dracort_b200.format import quantize as Q

    rng = np.random.default_rng(9)
    n, k = 48, 512
    first = Q.encode(14, Q.random_weight(rng, n, k)).reshape(-1, 210)
    last = np.concatenate([first[:, 2:], first[:, :2]], axis=1)  # llama.cpp order: d at bytes 208:210
    p = tmp_path / "q6.gguf"
    write_gguf(str(p), [("w", 14, (n, k), last.tobytes())], {"general.architecture": "llama"})
    w = load_gguf(str(p), "cuda")["w"]  # d_last is the default
    got = G.dequantize(14, w.tiled, n, k, layout="tiled").cpu().numpy()
    assert np.array_equal(got, O.dequantize_matrix(14, last.reshape(n, -1), n, k, q6k_order="d_last"))


def test_backend_loads_a_gguf_model_and_matches_the_oracle():
    import torch.nn as nn

    from dracort_b200.quantization import GGUFBackend, GGUFLinear

    class Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(256, 256, bias=False)
            self.k_proj = nn.Linear(256, 256, bias=False)
            self.v_proj = nn.Linear(256, 256, bias=False)

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = Attn()

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.model = nn.Module()
            self.model.layers = nn.ModuleList([Layer()])

    m = GGUFBackend(12).load_quantized_weights(TINY, Model(), {"q6k_order": "d_first"}, torch.device("cuda"))
    assert m._gguf_replaced == 3
    attn = m.model.layers[0].self_attn
    x = np.random.default_rng(1).standard_normal((3, 256)).astype(np.float32)
    with GGUFFile(TINY) as gf:
        for mod, gname in ((attn.q_proj, "blk.0.attn_q.weight"), (attn.k_proj, "blk.0.attn_k.weight"),
                           (attn.v_proj, "blk.0.attn_v.weight")):
            assert isinstance(mod, GGUFLinear)
            t = gf.tensor(gname)
            want = O.linear(x, t.ggml_type, gf.payload(gname).reshape(t.n_rows, -1), t.n_rows, t.k)
            got = mod(torch.from_numpy(x).cuda()).cpu().numpy()
            assert O.rel_l2(got, want) < 1e-3, gname
