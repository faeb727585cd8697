"""Host-side logic that needs no GPU: encoders, C-ABI loading and arguments, plugin API."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from dracort_b200 import _native as N
from dracort_b200.exceptions import DracoFormatError, KernelError
from dracort_b200.format import quantize as Q
from dracort_b200.format.gguf_types import BLOCK_LAYOUTS, packed_nbytes
from oracle import gguf_oracle as O

ROOT = Path(__file__).resolve().parents[1]


# ---------------------------------------------------------------- encoders
def test_q8_0_encoder_is_byte_identical_to_reference_test_encoder(golden):
    assert np.array_equal(Q.encode_q8_0(golden["q8_0_enc_w"]), golden["q8_0_enc_packed"])


@pytest.mark.parametrize("qtype,tol", [(2, 0.12), (3, 0.1), (6, 0.06), (7, 0.05), (8, 0.01), (12, 0.12), (13, 0.06),
                                      (14, 0.04)])
def test_encoders_round_trip_through_reference_decoder(qtype, tol):
    rng = np.random.default_rng(qtype)
    w = Q.random_weight(rng, 32, 1024)
    packed = Q.encode(qtype, w)
    assert packed.nbytes == packed_nbytes(qtype, 32, 1024)
    assert O.rel_l2(O.dequantize_matrix(qtype, packed, 32, 1024), w) < tol


def test_q6k_reorder_round_trip():
    rng = np.random.default_rng(1)
    p = Q.encode_q6_k(Q.random_weight(rng, 4, 512), order="d_first")
    last = Q.q6k_reorder(p, "d_first", "d_last")
    assert np.array_equal(Q.encode_q6_k(Q.random_weight(np.random.default_rng(1), 4, 512), order="d_last"), last)
    assert np.array_equal(Q.q6k_reorder(last, "d_last", "d_first"), p)
    a = O.dequantize_matrix(14, p, 4, 512)
    b = O.dequantize_matrix(14, last, 4, 512, q6k_order="d_last")
    assert np.array_equal(a, b)


def test_encoders_reject_bad_shapes():
    with pytest.raises(ValueError):
        Q.encode_q4_k(np.zeros((2, 100), np.float32))
    with pytest.raises(ValueError):
        Q.encode_q8_0(np.zeros((2, 33), np.float32))


# ---------------------------------------------------------------- C ABI
def _header_symbols():
    text = (ROOT / "include" / "draco_gguf.h").read_text()
    return sorted(set(re.findall(r"\b(draco_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = N.load()
    declared = _header_symbols()
    assert declared, "no declarations parsed"
    assert sorted(N.EXPORTED_SYMBOLS) == declared
    for s in declared:
        assert hasattr(lib, s), s
    assert N.version().startswith("draco_gguf")


def test_size_queries_need_no_gpu():
    lib = N.load()
    assert lib.draco_gguf_packed_bytes(12, 11008, 4096) == 11008 * 16 * 144
    assert lib.draco_gguf_packed_bytes(12, 10, 100) == -1
    assert lib.draco_gguf_tiled_bytes(12, 4096, 4096) == 4096 * 16 * 144
    # ragged rows pad to 16, Q8_0 rows pad to 256 elements
    assert lib.draco_gguf_tiled_bytes(14, 17, 512) == 32 * 2 * 210
    assert lib.draco_gguf_tiled_bytes(8, 16, 32 * 13) == 16 * 2 * 8 * 34
    assert lib.draco_gguf_tiled_bytes(13, 4096, 4096) == 4096 * 16 * 176
    # the 32-element types pad rows to 16 and k to 256 like Q8_0
    assert lib.draco_gguf_tiled_bytes(2, 17, 32 * 13) == 32 * 2 * 8 * 18
    assert lib.draco_gguf_tiled_bytes(7, 4096, 4096) == 4096 * 16 * 8 * 24
    assert lib.draco_gguf_packed_bytes(3, 10, 96) == 10 * 3 * 20
    assert lib.draco_gguf_packed_bytes(6, 10, 100) == -1
    bs, bb = ctypes.c_int(), ctypes.c_int()
    for qt in (2, 3, 6, 7, 8, 12, 13, 14):
        assert lib.draco_gguf_block_geometry(qt, ctypes.byref(bs), ctypes.byref(bb)) == 0
        assert (bs.value, bb.value) == BLOCK_LAYOUTS[qt]


def test_argument_errors_map_to_reference_exceptions():
    lib = N.load()
    with pytest.raises(DracoFormatError):  # unsupported type, like gguf.py:284-289
        N.check(lib.draco_gguf_dequant(16, 0, None, None, 1, 32, None))
    with pytest.raises(DracoFormatError):  # k not a multiple of the block, like gguf.py:291-296
        N.check(lib.draco_gguf_dequant(12, 0, None, None, 1, 100, None))
    with pytest.raises(ValueError):  # misaligned TILED pointer
        N.check(lib.draco_gguf_dequant(12, 2, 0x1001, 0x2000, 1, 256, None))
    arr = (N.GemvProblem * 1)()
    arr[0].qtype = 12
    arr[0].n_rows, arr[0].k, arr[0].ldx, arr[0].ldy = 16, 256, 256, 16
    arr[0].w, arr[0].x, arr[0].y = 0x1000, 0x2000, 0x3000
    with pytest.raises(ValueError):  # batch outside 1..32
        N.check(lib.draco_gguf_gemv_grouped(arr, 1, 33, None, 0, None))
    with pytest.raises(ValueError):  # no workspace
        N.check(lib.draco_gguf_gemv_grouped(arr, 1, 1, None, 0, None))
    assert "workspace" in N.last_error()
    assert lib.draco_gguf_gemv_workspace_bytes(arr, 1, 4) > 0
    assert lib.draco_gguf_gemv_workspace_bytes(arr, 1, 0) == 0
    with pytest.raises(KernelError):
        N.check(N.DRACO_ERR_TIMEOUT, "device wait ran out")


# ---------------------------------------------------------------- plugin API
def test_registry_contract():
    from dracort_b200.quantization import QUANT_REGISTRY, QuantizationRegistry, register_into

    assert {"gguf_q4_0", "gguf_q4_1", "gguf_q5_0", "gguf_q5_1", "gguf_q8_0", "gguf_q4_k", "gguf_q5_k", "gguf_q6_k",
            "gguf_q6_k_dlast"} <= set(QUANT_REGISTRY.list_methods())
    assert QUANT_REGISTRY.get("GGUF_Q4_K").name == "gguf_q4_k"
    assert "gguf_q8_0" in QUANT_REGISTRY and len(QUANT_REGISTRY) >= 4
    with pytest.raises(ValueError, match="gguf_q4_k"):  # names what is registered
        QUANT_REGISTRY.get("nope")
    assert QUANT_REGISTRY.detect_from_config({"quant_method": "awq"}) is None
    assert QUANT_REGISTRY.detect_from_config({}) is None
    assert QUANT_REGISTRY.detect_from_config({"quant_method": "GGUF_Q6_K"}) == "gguf_q6_k"

    class Foreign:  # any registry with register(name, backend), e.g. draco's QUANT_REGISTRY
        def __init__(self):
            self.d = {}

        def register(self, name, backend):
            self.d[name] = backend

    f = Foreign()
    assert sorted(register_into(f)) == sorted(f.d)
    r = QuantizationRegistry()
    register_into(r)
    assert r.get("gguf_q6_k_dlast").q6k_order == "d_last"
    # re-registering replaces the entry (with a warning), case-insensitively
    first = r.get("gguf_q8_0")
    register_into(r)
    assert r.get("GGUF_Q8_0") is not first and len(r) == 9


def test_backend_host_logic():
    from dracort_b200.quantization import GGUFBackend
    from dracort_b200.quantization.gguf import infer_k

    be = GGUFBackend(12)
    assert be.supported_bits == [4] and be.supported_schemes == ["weight_only"]
    assert be.estimate_memory(4096 * 4096) == 4096 * 16 * 144
    assert infer_k(12, 2304) == 4096 and infer_k(14, 9030) == 11008 and infer_k(8, 4352) == 4096
    with pytest.raises(DracoFormatError):
        infer_k(12, 100)
    with pytest.raises(DracoFormatError):
        GGUFBackend(10)  # Q2_K: decoded by the reference, no GPU kernel here
    assert GGUFBackend(2).supported_bits == [4] and GGUFBackend(7).name == "gguf_q5_1"
    assert not be.supports_gpu_kernel(torch.device("cpu"))
    with pytest.raises(ValueError, match="CUDA"):
        be.dequantize(torch.zeros((4, 144), dtype=torch.uint8))  # no CPU path
