"""The CPU oracle is pinned to the reference before anything is checked against it.

tests/golden/gguf_golden.npz was produced by the reference itself
(tests/golden/make_golden.py): draco.format.gguf._dequantize,
GenericGemmKernel.matmul_f32 (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K),
the reference tests' _enc_q8_0 and _ref_q4_k, and llama.cpp's gguf package for
the Q6_K d-last order (the same script checks that package's decode of the
Q4_0 / Q4_1 / Q5_0 / Q5_1 goldens against the reference's).
"""

import numpy as np
import pytest

from oracle import gguf_oracle as O

TYPES = [(2, "q4_0"), (3, "q4_1"), (6, "q5_0"), (7, "q5_1"), (8, "q8_0"), (12, "q4_k"), (13, "q5_k"), (14, "q6_k")]


def bits_equal(a, b):
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("qtype,name", TYPES)
def test_oracle_dequant_bit_exact_with_reference(golden, qtype, name):
    n, k = (int(v) for v in golden[f"{name}_shape"])
    got = O.dequantize_matrix(qtype, golden[f"{name}_packed"], n, k)
    assert bits_equal(got, golden[f"{name}_expected"])


def test_oracle_q4k_matches_reference_test_loop_decoder(golden):
    n, k = (int(v) for v in golden["q4_k_shape"])
    got = O.dequantize_matrix(12, golden["q4_k_packed"], n, k).reshape(-1, 256)[:8]
    assert bits_equal(got, golden["q4_k_loop_expected"])


def test_oracle_q6k_dlast_matches_llamacpp_gguf_package(golden):
    n, k = (int(v) for v in golden["q6_k_shape"])
    got = O.dequantize_matrix(14, golden["q6_k_dlast_packed"], n, k, q6k_order="d_last")
    assert bits_equal(got, golden["q6_k_dlast_expected"])


@pytest.mark.parametrize("qtype,name", TYPES)
def test_oracle_linear_matches_reference_matmul(golden, qtype, name):
    n, k = (int(v) for v in golden[f"{name}_shape"])
    y = O.linear(golden[f"{name}_lin_x"], qtype, golden[f"{name}_packed"], n, k)
    assert np.array_equal(y, golden[f"{name}_lin_y"])


def test_oracle_rejects_what_the_reference_rejects():
    with pytest.raises(O.OracleFormatError):
        O.dequantize(16, b"\x00" * 100, 32)  # unsupported type (gguf.py:284-289)
    with pytest.raises(O.OracleFormatError):
        O.dequantize(12, b"\x00" * 144, 100)  # n not a multiple of the block (gguf.py:291-296)


def test_planted_fifth_bit_mistake_is_caught(golden):
    """Reading the Q5_0 fifth bits in big-endian order must fail the golden check."""
    n, k = (int(v) for v in golden["q5_0_shape"])
    b = golden["q5_0_packed"].reshape(-1, 22).copy()
    b[:, 2:6] = b[:, 2:6][:, ::-1]
    got = O.dequantize_matrix(6, b, n, k)
    assert not bits_equal(got, golden["q5_0_expected"])


def test_planted_mistake_is_caught(golden):
    """A decoder that swaps nibble order must fail the golden check (the harness has teeth)."""
    n, k = (int(v) for v in golden["q4_k_shape"])
    b = golden["q4_k_packed"].reshape(-1, 144).copy()
    b[:, 16:144] = ((b[:, 16:144] & 0x0F) << 4) | (b[:, 16:144] >> 4)
    got = O.dequantize_matrix(12, b, n, k)
    assert not bits_equal(got, golden["q4_k_expected"])


def test_rel_l2():
    r = np.ones(10)
    assert O.rel_l2(r, r) == 0.0
    assert abs(O.rel_l2(r * 1.001, r) - 1e-3) < 1e-12
