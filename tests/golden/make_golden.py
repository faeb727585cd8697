"""Generate the golden parity fixtures in tests/golden/ from the REAL reference.

Run in a container where the reference (sadrasa97/DracoRT) is checked out:

    python tests/golden/make_golden.py --reference /path/to/DracoRT
    (or DRACO_REFERENCE=/path/to/DracoRT python tests/golden/make_golden.py)

The reference is imported the way its own tests do it (tests/conftest.py:18-29
stubs the top-level packages so that draco/__init__.py, which pulls in torch,
the server and transformers, is not executed).  Every expected output below is
produced by reference code:

* ``draco.format.gguf._dequantize`` (gguf.py:272-497) for Q8_0 / Q4_K / Q5_K /
  Q6_K and Q4_0 / Q4_1 / Q5_0 / Q5_1;
* ``GenericGemmKernel.matmul_f32`` (runtime/cpu/kernels/generic.py:32-33) for
  the linear-layer goldens;
* the reference test suite's own helpers (tests/format/test_gguf.py): the Q8_0
  encoder ``_enc_q8_0`` (:145-155) and the plain-loop Q4_K decoder
  ``_ref_q4_k`` (:287-301);
* llama.cpp's ``gguf`` Python package (0.19.0, if installed) for the Q6_K
  d-last byte order used in real .gguf files.

The fixtures are small .npz files; nothing at test time reads the reference.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = None  # the reference checkout, from --reference or DRACO_REFERENCE (required)


def _stub(name: str, path: Path) -> None:
    if name not in sys.modules:
        m = types.ModuleType(name)
        m.__path__ = [str(path)]
        sys.modules[name] = m


def load_reference():
    if REF is None:
        raise SystemExit("give the reference checkout: --reference PATH or DRACO_REFERENCE=PATH")
    d = REF / "draco"
    if not d.is_dir():
        raise SystemExit(f"reference not found at {REF}")
    for name, sub in [
        ("draco", ""),
        ("draco.format", "format"),
        ("draco.runtime", "runtime"),
        ("draco.runtime.cpu", "runtime/cpu"),
        ("draco.runtime.cpu.kernels", "runtime/cpu/kernels"),
        ("draco.quantization", "quantization"),
        ("draco.utils", "utils"),
    ]:
        _stub(name, d / sub)
    import draco.format.gguf as gguf  # noqa: E402
    from draco.runtime.cpu.kernels.generic import GenericGemmKernel  # noqa: E402

    spec = importlib.util.spec_from_file_location("ref_test_gguf", REF / "tests" / "format" / "test_gguf.py")
    tmod = importlib.util.module_from_spec(spec)
    _stub("draco.format", d / "format")
    spec.loader.exec_module(tmod)
    return gguf, GenericGemmKernel(), tmod


def finite_f16(rng, n, lo_exp=-20, hi_exp=2, with_edges=True):
    """Finite fp16 values (normal, subnormal, zero, negative) as float32."""
    mant = rng.uniform(1.0, 2.0, n)
    e = rng.integers(lo_exp, hi_exp, n)
    sign = np.where(rng.random(n) < 0.3, -1.0, 1.0)
    v = (sign * mant * np.exp2(e)).astype(np.float16)
    if with_edges and n >= 6:
        v[:6] = np.array([0.0, -0.0, 6e-8, 5.96e-08, 65504.0, -0.000061], dtype=np.float16)
    return v


def random_blocks(rng, qtype, nb):
    """Random bytes for every field except the fp16 scales, which are finite."""
    if qtype == 8:
        b = rng.integers(0, 256, (nb, 34), dtype=np.uint8)
        b[:, 0:2] = finite_f16(rng, nb).view(np.uint8).reshape(nb, 2)
    elif qtype in (12, 13):
        b = rng.integers(0, 256, (nb, 144 if qtype == 12 else 176), dtype=np.uint8)
        b[:, 0:2] = finite_f16(rng, nb).view(np.uint8).reshape(nb, 2)
        b[:, 2:4] = finite_f16(rng, nb).view(np.uint8).reshape(nb, 2)
    elif qtype in (2, 3, 6, 7):
        b = rng.integers(0, 256, (nb, {2: 18, 3: 20, 6: 22, 7: 24}[qtype]), dtype=np.uint8)
        b[:, 0:2] = finite_f16(rng, nb).view(np.uint8).reshape(nb, 2)
        if qtype in (3, 7):  # m
            b[:, 2:4] = finite_f16(rng, nb).view(np.uint8).reshape(nb, 2)
    else:
        b = rng.integers(0, 256, (nb, 210), dtype=np.uint8)
        b[:, 0:2] = finite_f16(rng, nb).view(np.uint8).reshape(nb, 2)
    return b


def main() -> None:
    gguf, kern, tmod = load_reference()
    rng = np.random.default_rng(20261201)
    out = {}

    # ---- per-type dequantization goldens (random bytes, reference decode) ----
    for qtype, name, (bs, bb) in [(8, "q8_0", (32, 34)), (12, "q4_k", (256, 144)), (14, "q6_k", (256, 210))]:
        n_rows, k = 6, 4 * bs * (8 if bs == 32 else 1)
        nb = n_rows * k // bs
        blocks = random_blocks(rng, qtype, nb)
        expected = gguf._dequantize(qtype, blocks.tobytes(), n_rows * k)
        out[f"{name}_packed"] = blocks.reshape(n_rows, -1)
        out[f"{name}_shape"] = np.array([n_rows, k])
        out[f"{name}_expected"] = expected.reshape(n_rows, k).astype(np.float32)

    # ---- Q4_K: the reference tests' independent plain-loop decoder ----
    q4 = out["q4_k_packed"].reshape(-1, 144)
    loop = []
    for blk in q4[:8]:
        d = float(np.frombuffer(blk[0:2].tobytes(), dtype=np.float16)[0])
        dmin = float(np.frombuffer(blk[2:4].tobytes(), dtype=np.float16)[0])
        loop.append(tmod._ref_q4_k(np.float32(d), np.float32(dmin), blk[4:16], blk[16:144]))
    out["q4_k_loop_expected"] = np.stack(loop).astype(np.float32)

    # ---- Q6_K d-last (real .gguf order) through llama.cpp's gguf package ----
    q6 = out["q6_k_packed"].reshape(-1, 210)
    dlast = np.concatenate([q6[:, 2:210], q6[:, 0:2]], axis=1)
    out["q6_k_dlast_packed"] = dlast.reshape(out["q6_k_packed"].shape)
    try:
        import gguf as gguf_pkg
        from gguf import GGMLQuantizationType

        pkg = gguf_pkg.quants.dequantize(dlast.reshape(out["q6_k_packed"].shape), GGMLQuantizationType.Q6_K)
        out["q6_k_dlast_expected"] = np.asarray(pkg, dtype=np.float32).reshape(out["q6_k_expected"].shape)
        out["q6_k_dlast_source"] = np.array("gguf-0.19.0")
    except Exception as e:  # pragma: no cover
        print("gguf package unavailable:", e)

    # ---- Q8_0 encoder parity with the reference test encoder ----
    w = (rng.standard_normal((4, 256)) * 0.02).astype(np.float32)
    out["q8_0_enc_w"] = w
    out["q8_0_enc_packed"] = np.frombuffer(tmod._enc_q8_0(w.reshape(-1)), dtype=np.uint8).reshape(4, -1)

    # ---- linear-layer goldens: _dequantize + GenericGemmKernel.matmul_f32 ----
    for qtype, name in [(8, "q8_0"), (12, "q4_k"), (14, "q6_k")]:
        packed = out[f"{name}_packed"]
        n_rows, k = out[f"{name}_shape"]
        w = gguf._dequantize(qtype, packed.tobytes(), int(n_rows * k)).reshape(n_rows, k)
        x = rng.standard_normal((3, int(k))).astype(np.float32)
        out[f"{name}_lin_x"] = x
        out[f"{name}_lin_y"] = kern.matmul_f32(x, w).astype(np.float32)

    # ---- Q5_K (own stream, so the keys above keep their bytes) ----
    rng5 = np.random.default_rng(20261202)
    n_rows, k = 6, 1024
    blocks = random_blocks(rng5, 13, n_rows * k // 256)
    out["q5_k_packed"] = blocks.reshape(n_rows, -1)
    out["q5_k_shape"] = np.array([n_rows, k])
    w5 = gguf._dequantize(13, blocks.tobytes(), n_rows * k).reshape(n_rows, k)
    out["q5_k_expected"] = w5.astype(np.float32)
    x5 = rng5.standard_normal((3, k)).astype(np.float32)
    out["q5_k_lin_x"] = x5
    out["q5_k_lin_y"] = kern.matmul_f32(x5, w5).astype(np.float32)

    # ---- Q4_0 / Q4_1 / Q5_0 / Q5_1 (own stream; k = 320 leaves a ragged
    # tail super-block of two 32-element blocks) ----
    rngl = np.random.default_rng(20261203)
    for qtype, name in [(2, "q4_0"), (3, "q4_1"), (6, "q5_0"), (7, "q5_1")]:
        n_rows, k = 6, 320
        blocks = random_blocks(rngl, qtype, n_rows * k // 32)
        wl = gguf._dequantize(qtype, blocks.tobytes(), n_rows * k).reshape(n_rows, k)
        out[f"{name}_packed"] = blocks.reshape(n_rows, -1)
        out[f"{name}_shape"] = np.array([n_rows, k])
        out[f"{name}_expected"] = wl.astype(np.float32)
        xl = rngl.standard_normal((3, k)).astype(np.float32)
        out[f"{name}_lin_x"] = xl
        out[f"{name}_lin_y"] = kern.matmul_f32(xl, wl).astype(np.float32)
        try:  # second opinion: llama.cpp's own decoder
            import gguf as gguf_pkg
            from gguf import GGMLQuantizationType

            pkg = gguf_pkg.quants.dequantize(blocks.reshape(n_rows, -1), GGMLQuantizationType(qtype))
            same = np.array_equal(np.asarray(pkg, np.float32).reshape(n_rows, k).view(np.uint32),
                                  wl.astype(np.float32).view(np.uint32))
            print(f"{name}: reference decode {'==' if same else '!='} gguf package decode")
        except Exception as e:  # pragma: no cover
            print("gguf package unavailable:", e)

    path = HERE / "gguf_golden.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size} bytes), keys: {sorted(out)}")


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="regenerate tests/golden/gguf_golden.npz from the reference")
    ap.add_argument("--reference", default=os.environ.get("DRACO_REFERENCE"),
                    help="path of the DracoRT checkout (default: $DRACO_REFERENCE)")
    REF = Path(ap.parse_args().reference) if ap.parse_args().reference else None
    main()
