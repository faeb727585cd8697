"""Synthetic workloads with the benchmark configurations' shapes.

* Config 1 — Q8_0 GEMV, W 4096x4096, x fp32 [1, 4096].
* Config 2 — Q4_K decode GEMV over one Llama-7B-shaped decoder layer's seven
  projections (q, k, v, o 4096x4096; gate, up 11008x4096; down 4096x11008),
  x fp32 at batch 1, 4, 16.
* Config 3 — mixed Q4_K/Q6_K prefill dequant-GEMM, M = 2048 tokens: gate and
  up 11008x4096 in Q4_K, down 4096x11008 in Q6_K, bf16 activations.
* Config 4 — the same projections in Q4_K_M (Q6_K for v and down).
  Config 4's model step runs the 32 layers' projections back to back.
* Config 5 — Mixtral-8x7B-shaped MoE FFN: 8 Q4_K experts (gate/up
  14336x4096, down 4096x14336), top-2 routing, 256 bf16 tokens.

Weights are drawn from N(0, 0.02) with a recorded seed and encoded with the
synthetic GGUF encoders (dracort_b200.format.quantize); activations from
N(0, 1).  Algorithmic bytes count the packed weights plus fp32 x and y once.
"""

from __future__ import annotations

import functools
from dataclasses import dataclass
from typing import List, Sequence, Tuple

import numpy as np

from dracort_b200.format.gguf_types import (
    GGML_TYPE_Q4_K,
    GGML_TYPE_Q6_K,
    GGML_TYPE_Q8_0,
    packed_nbytes,
)
from dracort_b200.format.quantize import encode, random_weight

HIDDEN = 4096
FFN = 11008

#: (name, n_rows = out_features, k = in_features) of one Llama-7B decoder layer
LLAMA7B_PROJECTIONS: Tuple[Tuple[str, int, int], ...] = (
    ("q_proj", HIDDEN, HIDDEN),
    ("k_proj", HIDDEN, HIDDEN),
    ("v_proj", HIDDEN, HIDDEN),
    ("o_proj", HIDDEN, HIDDEN),
    ("gate_proj", FFN, HIDDEN),
    ("up_proj", FFN, HIDDEN),
    ("down_proj", HIDDEN, FFN),
)


@dataclass
class WeightSpec:
    name: str
    qtype: int
    n_rows: int
    k: int

    @property
    def nbytes(self) -> int:
        return packed_nbytes(self.qtype, self.n_rows, self.k)


def layer_specs(mix: str = "q4_k") -> List[WeightSpec]:
    """Projection specs of one decoder layer: 'q4_k' (config 2) or 'q4_k_m' (config 4)."""
    out = []
    for name, n, k in LLAMA7B_PROJECTIONS:
        qt = GGML_TYPE_Q4_K
        if mix == "q4_k_m" and name in ("v_proj", "down_proj"):
            qt = GGML_TYPE_Q6_K
        elif mix not in ("q4_k", "q4_k_m"):
            raise ValueError(f"unknown mix {mix!r}")
        out.append(WeightSpec(name, qt, n, k))
    return out


PREFILL_TOKENS = 2048


def prefill_specs(mix: str = "mixed") -> List[WeightSpec]:
    """Config 3: gate/up (Q4_K) and down (Q6_K) of one layer; 'q4'/'q6' make all three one type."""
    qt_gu = GGML_TYPE_Q6_K if mix == "q6" else GGML_TYPE_Q4_K
    qt_d = GGML_TYPE_Q4_K if mix == "q4" else GGML_TYPE_Q6_K
    return [WeightSpec("gate_proj", qt_gu, FFN, HIDDEN), WeightSpec("up_proj", qt_gu, FFN, HIDDEN),
            WeightSpec("down_proj", qt_d, HIDDEN, FFN)]


def prefill_flops(specs: Sequence[WeightSpec], m: int = PREFILL_TOKENS) -> int:
    return sum(2 * m * s.n_rows * s.k for s in specs)


MODEL_LAYERS = 32


def model_layers(seed: int, n_layers: int = MODEL_LAYERS, mix: str = "q4_k_m"):
    """Config 4: packed projections of an n-layer Llama-7B-shaped model.  One
    layer is encoded from seeded N(0, 0.02) weights; every other layer's
    projections are seeded row permutations of its packed rows (each row a
    valid quantized N(0, 0.02) row).  Returns (specs, [layer][projection] packed).
    The last result is kept (the 32-layer step and the decode-step benchmark
    use the same model); callers must not modify the arrays."""
    return _model_layers(int(seed), int(n_layers), str(mix))


@functools.lru_cache(maxsize=1)
def _model_layers(seed: int, n_layers: int, mix: str):
    specs = layer_specs(mix)
    base = encode_specs(specs, seed)
    rng = np.random.default_rng(seed + 1)
    layers = [base] + [[p[rng.permutation(s.n_rows)] for s, p in zip(specs, base)] for _ in range(n_layers - 1)]
    return specs, layers


MOE_EXPERTS, MOE_HIDDEN, MOE_FFN, MOE_TOP_K, MOE_TOKENS = 8, 4096, 14336, 2, 256


def moe_experts(seed: int, n_exp: int = MOE_EXPERTS, hidden: int = MOE_HIDDEN, ffn: int = MOE_FFN,
                qtype: int = GGML_TYPE_Q4_K):
    """Config-5 experts: (qtype, gate, up, down) packed payloads.  One expert is
    encoded from seeded N(0, 0.02) weights; the others are seeded row
    permutations of its packed rows (each row a valid quantized N(0, 0.02)
    row), which keeps the set distinct without encoding 1.4 G weights."""
    rng = np.random.default_rng(seed)
    base = (encode(qtype, random_weight(rng, ffn, hidden)), encode(qtype, random_weight(rng, ffn, hidden)),
            encode(qtype, random_weight(rng, hidden, ffn)))
    out = [(qtype,) + base]
    for _ in range(1, n_exp):
        out.append((qtype, base[0][rng.permutation(ffn)], base[1][rng.permutation(ffn)],
                    base[2][rng.permutation(hidden)]))
    return out


def q8_0_spec() -> List[WeightSpec]:
    return [WeightSpec("w", GGML_TYPE_Q8_0, 4096, 4096)]


def encode_specs(specs: Sequence[WeightSpec], seed: int) -> List[np.ndarray]:
    """Seeded N(0, 0.02) weights encoded per spec (packed uint8 arrays)."""
    rng = np.random.default_rng(seed)
    return [encode(s.qtype, random_weight(rng, s.n_rows, s.k)) for s in specs]


def algorithmic_bytes(specs: Sequence[WeightSpec], batch: int) -> int:
    """Packed weights + fp32 activations in + fp32 outputs, each counted once."""
    return sum(s.nbytes + 4 * batch * (s.k + s.n_rows) for s in specs)


def flops(specs: Sequence[WeightSpec], batch: int) -> int:
    return sum(2 * batch * s.n_rows * s.k for s in specs)
