"""GPU decode step for GGUF llama-family models (dracort_b200.gguf_executor)
against the reference executor's logits on three fixtures
(tests/golden/make_decode_golden.py): tiny_llama_decode.gguf (every GPU block
type), tiny_qwen2_decode.gguf (q/k/v and o_proj biases, tied embeddings,
rope base 1e6) and tiny_fused_decode.gguf (a fused q/k/v weight, gate/up/down
biases), and against the pinned decode oracle.

Bar: the decode GEMV's 1e-3 relative L2 per projection, carried through two
layers and the output head: logits within 2e-3 relative L2, and the greedy
tokens identical."""

from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from dracort_b200.format.gguf_file import GGUFFile  # noqa: E402
from dracort_b200.gguf_executor import GPUExecutionBackend  # noqa: E402
from oracle.llama_decode import OracleLlama  # noqa: E402

HERE = Path(__file__).resolve().parent / "golden"
FIXTURES = ["tiny_llama_decode", "tiny_qwen2_decode", "tiny_fused_decode"]
TOL = 2e-3


@pytest.fixture(scope="module", params=FIXTURES)
def name(request):
    return request.param


@pytest.fixture(scope="module")
def ref(name):
    return np.load(HERE / f"{name}_ref.npz")


@pytest.fixture(scope="module")
def backend(name):
    return GPUExecutionBackend(str(HERE / f"{name}.gguf"), max_num_seqs=4, q6k_order="d_first")


def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_prefill_logits_of_every_position(backend, ref):
    s = backend.new_sequence()
    try:
        got = backend.forward_step(s, ref["prompt"], 0, return_all_positions=True)
    finally:
        backend.end_sequence(s)
    assert got.shape == ref["prefill_logits"].shape
    assert rel(got, ref["prefill_logits"]) < TOL


def test_greedy_decode_tokens_and_logits(backend, ref):
    s = backend.new_sequence()
    try:
        ids = list(ref["prompt"])
        logits = backend.forward_step(s, np.array(ids), 0)
        for t_ref, l_ref in zip(ref["decode_tokens"], ref["decode_logits"]):
            t = int(np.argmax(logits))
            assert t == int(t_ref)
            ids.append(t)
            logits = backend.forward_step(s, np.array([t]), len(ids) - 1)
            assert rel(logits, l_ref) < TOL
    finally:
        backend.end_sequence(s)


def test_generate_greedy(backend, ref):
    out = backend.generate_greedy(list(ref["prompt"]), len(ref["decode_tokens"]))
    assert out == list(ref["prompt"]) + [int(t) for t in ref["decode_tokens"]]


def test_one_token_pass_launches(backend):
    """A one-token pass starts five library kernels per layer: the q/k/v,
    o_proj, gate/up and down GEMVs (RMSNorm scales computed inside at batch
    1) and the attention with RoPE and the cache append inside."""
    assert backend.launches_per_layer == 5


def test_batch_decode_of_two_sequences(backend, ref):
    sa, sb = backend.new_sequence(), backend.new_sequence()
    try:
        la = backend.forward_step(sa, ref["prompt"], 0)
        lb = backend.forward_step(sb, ref["prompt_b"], 0)
        toks = [int(np.argmax(la)), int(np.argmax(lb))]
        assert toks == [int(t) for t in ref["batch_tokens"]]
        got = backend.forward_batch_decode([sa, sb], toks, [len(ref["prompt"]), len(ref["prompt_b"])])
        assert rel(got, ref["batch_logits"]) < TOL
    finally:
        backend.end_sequence(sa)
        backend.end_sequence(sb)


def test_long_prompt_in_chunks_matches_oracle(backend, name):
    """60 tokens (the fixture's context is 64): chunks of rows through the
    GEMV, each attending to the cache the earlier chunks wrote."""
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, backend.config.vocab_size, 40)
    gf = GGUFFile(str(HERE / f"{name}.gguf"))
    try:
        orc = OracleLlama(gf, q6k_order="d_first")
    finally:
        gf.close()
    so, s = orc.new_sequence(), backend.new_sequence()
    try:
        ref_all = orc.forward_step(so, prompt, 0, return_all_positions=True)
        got_all = backend.forward_step(s, prompt, 0, return_all_positions=True)
        assert rel(got_all, ref_all) < TOL
        more = rng.integers(0, backend.config.vocab_size, 20)
        assert rel(backend.forward_step(s, more, 40, return_all_positions=True),
                   orc.forward_step(so, more, 40, return_all_positions=True)) < TOL
    finally:
        backend.end_sequence(s)


def test_sequence_bookkeeping_and_argument_errors(backend):
    seqs = [backend.new_sequence() for _ in range(backend.max_num_seqs)]
    with pytest.raises(RuntimeError):
        backend.new_sequence()  # every cache slot in use
    backend.end_sequence(seqs.pop())
    s = backend.new_sequence()
    seqs.append(s)
    with pytest.raises(ValueError):
        backend.forward_step(s, np.array([1, 2]), 3)  # must continue the cached positions
    with pytest.raises(ValueError):
        backend.forward_step(s, np.array([backend.config.vocab_size]), 0)  # outside the vocabulary
    backend.forward_step(s, np.array([1, 2, 3]), 0)
    backend.truncate_sequence(s, 1)
    backend.forward_step(s, np.array([4]), 1)
    for q in seqs:
        backend.end_sequence(q)
