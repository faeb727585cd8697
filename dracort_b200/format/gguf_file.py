"""GGUF container: a memory-mapped reader and a minimal writer.

Replaces the parsing half of draco/format/gguf.py's ``GGUFReader``
(gguf.py:528-662: header, metadata key/values, tensor infos, data offset) and
its ``GgufTensorInfo`` (gguf.py:504-520).  The reader hands out zero-copy
uint8 views of the packed payloads; nothing is dequantized on the host (the
reference's ``get_tensor`` turns every weight into a 4-byte-per-weight fp32
cache, gguf.py:820-834; here the packed bytes go to the GPU as they are, see
``dracort_b200.gguf_loader``).

File layout (the GGUF specification, versions 1-3, little-endian):

    magic "GGUF" | version u32 | tensor_count u64 | kv_count u64
    kv_count  x  (key: string, value_type: u32, value)
    tensor_count x (name: string, n_dims: u32, dims: u64[n_dims], ggml_type: u32, offset: u64)
    padding to `general.alignment` (default 32), then the tensor data; each
    tensor's offset is relative to the start of the data section.

A string is a u64 byte length followed by UTF-8 bytes; an array value is an
element type (u32), a count (u64) and the elements.  ``dims`` run from the
fastest-varying dimension (GGML ne0, the reduction length of a weight) to the
slowest, so a weight [n_rows, k] is stored as dims (k, n_rows); ``shape`` here
is the reversed, row-major order (gguf.py:651-653 does the same).
"""

from __future__ import annotations

import mmap
import os
import re
import struct
from dataclasses import dataclass
from typing import Any, Dict, Iterator, List, Mapping, Optional, Sequence, Tuple

import numpy as np

from dracort_b200.exceptions import DracoFormatError
from dracort_b200.format.gguf_types import BLOCK_LAYOUTS, GGML_TYPE_BF16, GGML_TYPE_F16, GGML_TYPE_F32

GGUF_MAGIC = b"GGUF"
GGML_TYPE_F64 = 28
DEFAULT_ALIGNMENT = 32

# metadata value types (GGUF specification)
VT_UINT8, VT_INT8, VT_UINT16, VT_INT16, VT_UINT32, VT_INT32, VT_FLOAT32 = 0, 1, 2, 3, 4, 5, 6
VT_BOOL, VT_STRING, VT_ARRAY, VT_UINT64, VT_INT64, VT_FLOAT64 = 7, 8, 9, 10, 11, 12
_SCALAR_FMT = {VT_UINT8: "<B", VT_INT8: "<b", VT_UINT16: "<H", VT_INT16: "<h", VT_UINT32: "<I",
               VT_INT32: "<i", VT_FLOAT32: "<f", VT_BOOL: "<?", VT_UINT64: "<Q", VT_INT64: "<q",
               VT_FLOAT64: "<d"}

# element bytes of the dense types; quantized types use BLOCK_LAYOUTS
_DENSE_BYTES = {GGML_TYPE_F32: 4, GGML_TYPE_F16: 2, GGML_TYPE_BF16: 2, GGML_TYPE_F64: 8}


@dataclass(frozen=True)
class GGUFTensor:
    """One tensor of a GGUF file (the fields of the reference's GgufTensorInfo
    that describe the payload: name, ggml_type, row-major shape, absolute file
    offset, payload bytes)."""

    name: str
    ggml_type: int
    shape: Tuple[int, ...]
    offset: int
    nbytes: int
    alignment: int = DEFAULT_ALIGNMENT

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    @property
    def k(self) -> int:
        """Reduction length (GGML ne0): the last dimension of the row-major shape."""
        return self.shape[-1] if self.shape else 1

    @property
    def n_rows(self) -> int:
        return self.n_elements // self.k if self.k else 0

    @property
    def is_quantized(self) -> bool:
        return self.ggml_type in BLOCK_LAYOUTS


def tensor_nbytes(ggml_type: int, shape: Sequence[int]) -> int:
    """Payload bytes of a tensor; quantized rows must hold whole blocks."""
    n = 1
    for d in shape:
        n *= int(d)
    if ggml_type in _DENSE_BYTES:
        return n * _DENSE_BYTES[ggml_type]
    if ggml_type in BLOCK_LAYOUTS:
        bs, bb = BLOCK_LAYOUTS[ggml_type]
        k = int(shape[-1]) if len(shape) else 1
        if k % bs:
            raise DracoFormatError(f"row length {k} is not a multiple of block size {bs} for ggml type {ggml_type}")
        return n // bs * bb
    raise DracoFormatError(f"ggml type {ggml_type} is not supported (dense F32/F16/BF16/F64, or "
                           f"quantized {sorted(BLOCK_LAYOUTS)})")


class _Cursor:
    """Bounds-checked little-endian reads from a buffer."""

    def __init__(self, buf, pos: int, end: int, path: str) -> None:
        self.buf, self.pos, self.end, self.path = buf, pos, end, path

    def take(self, n: int) -> int:
        if n < 0 or self.pos + n > self.end:
            raise DracoFormatError(f"truncated GGUF header in '{self.path}' (needs byte {self.pos + n}, "
                                   f"file has {self.end})")
        p = self.pos
        self.pos += n
        return p

    def scalar(self, fmt: str):
        return struct.unpack_from(fmt, self.buf, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.scalar("<Q")
        p = self.take(n)
        try:
            return bytes(self.buf[p:p + n]).decode("utf-8")
        except UnicodeDecodeError as e:
            raise DracoFormatError(f"GGUF string at byte {p} of '{self.path}' is not UTF-8") from e

    def value(self, vtype: int, depth: int = 0) -> Any:
        if vtype == VT_STRING:
            return self.string()
        if vtype == VT_ARRAY:
            if depth > 4:
                raise DracoFormatError(f"GGUF arrays nested too deeply in '{self.path}'")
            etype = self.scalar("<I")
            count = self.scalar("<Q")
            if etype in _SCALAR_FMT and etype != VT_BOOL:
                fmt = _SCALAR_FMT[etype]
                size = struct.calcsize(fmt)
                p = self.take(size * count)
                return np.frombuffer(bytes(self.buf[p:p + size * count]), dtype=np.dtype(fmt)).tolist()
            return [self.value(etype, depth + 1) for _ in range(count)]
        fmt = _SCALAR_FMT.get(vtype)
        if fmt is None:
            raise DracoFormatError(f"unknown GGUF metadata value type {vtype} in '{self.path}'")
        return self.scalar(fmt)


class GGUFFile:
    """Memory-mapped .gguf file: metadata, tensor index and zero-copy payload views.

    Mirrors the checks of GGUFReader.__init__ / _build_index (gguf.py:531-662):
    bad magic, unsupported version, invalid alignment, truncated header and
    tensors past the end of the file raise DracoFormatError."""

    def __init__(self, path: str) -> None:
        self.path = str(path)
        self._file = open(self.path, "rb")
        self._mmap = None
        try:
            size = os.fstat(self._file.fileno()).st_size
            if size < 24:
                raise DracoFormatError(f"'{self.path}' is too small to be a GGUF file ({size} bytes)")
            self._mmap = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
            self.file_size = size
            cur = _Cursor(self._mmap, 0, size, self.path)
            magic = bytes(self._mmap[cur.take(4):4])
            if magic != GGUF_MAGIC:
                raise DracoFormatError(f"'{self.path}' is not a GGUF file (magic {magic!r})")
            self.version = cur.scalar("<I")
            if self.version not in (1, 2, 3):
                raise DracoFormatError(f"GGUF version {self.version} of '{self.path}' is not supported (1-3)")
            n_tensors = cur.scalar("<Q")
            n_kv = cur.scalar("<Q")
            self.metadata: Dict[str, Any] = {}
            for _ in range(n_kv):
                key = cur.string()
                self.metadata[key] = cur.value(cur.scalar("<I"))
            align = self.metadata.get("general.alignment", DEFAULT_ALIGNMENT)
            if not isinstance(align, int) or align <= 0 or align % 8:
                raise DracoFormatError(f"invalid general.alignment {align!r} in '{self.path}' "
                                       f"(must be a positive multiple of 8)")
            self.alignment = align
            raw = []
            for _ in range(n_tensors):
                name = cur.string()
                n_dims = cur.scalar("<I")
                if n_dims > 8:
                    raise DracoFormatError(f"tensor '{name}' of '{self.path}' has {n_dims} dimensions")
                dims = [cur.scalar("<Q") for _ in range(n_dims)]
                raw.append((name, dims, cur.scalar("<I"), cur.scalar("<Q")))
            self.data_offset = -(-cur.pos // align) * align
            self.tensors: Dict[str, GGUFTensor] = {}
            for name, dims, ttype, rel in raw:
                if name in self.tensors:
                    raise DracoFormatError(f"duplicate tensor name '{name}' in '{self.path}'")
                shape = tuple(int(d) for d in reversed(dims))
                nbytes = tensor_nbytes(ttype, shape) if (ttype in _DENSE_BYTES or ttype in BLOCK_LAYOUTS) else -1
                off = self.data_offset + rel
                if nbytes >= 0 and off + nbytes > size:
                    raise DracoFormatError(f"tensor '{name}' extends past the end of '{self.path}' "
                                           f"({off}+{nbytes} > {size})")
                self.tensors[name] = GGUFTensor(name, ttype, shape, off, nbytes, align)
        except Exception:
            self.close()
            raise

    # -- index -----------------------------------------------------------
    @property
    def architecture(self) -> str:
        return str(self.metadata.get("general.architecture", ""))

    def tensor_names(self) -> List[str]:
        return list(self.tensors)

    def __iter__(self) -> Iterator[GGUFTensor]:
        return iter(self.tensors.values())

    def tensor(self, name: str) -> GGUFTensor:
        try:
            return self.tensors[name]
        except KeyError:
            raise KeyError(f"no tensor named '{name}' in '{self.path}'") from None

    def payload(self, name: str) -> np.ndarray:
        """Zero-copy uint8 view of a tensor's bytes (valid while the file is open)."""
        t = self.tensor(name)
        if t.nbytes < 0:
            raise DracoFormatError(f"tensor '{name}' has ggml type {t.ggml_type}, which this library cannot read")
        return np.frombuffer(self._mmap, dtype=np.uint8, count=t.nbytes, offset=t.offset)

    def canonical_names(self) -> Dict[str, str]:
        """GGUF name -> the HF-style name DracoRT's executor looks up, for
        llama-family architectures (the naming of gguf.py:104-171); other
        names map to themselves."""
        return {n: canonical_name(n) for n in self.tensors}

    # -- lifetime --------------------------------------------------------
    def close(self) -> None:
        if self._mmap is not None:
            try:
                self._mmap.close()
            except BufferError:  # a payload view is still alive; the map closes with it
                pass
            self._mmap = None
        if not self._file.closed:
            self._file.close()

    def __enter__(self) -> "GGUFFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


# llama-family GGUF tensor names -> HF-style module parameter names
_TOP_NAMES = {"token_embd.weight": "model.embed_tokens.weight", "output_norm.weight": "model.norm.weight",
              "output.weight": "model.lm_head.weight"}
_BLOCK_NAMES = {"attn_norm": "input_layernorm", "attn_q": "self_attn.q_proj", "attn_k": "self_attn.k_proj",
                "attn_v": "self_attn.v_proj", "attn_output": "self_attn.o_proj", "attn_qkv": "self_attn.qkv_proj",
                "ffn_norm": "post_attention_layernorm", "ffn_gate": "mlp.gate_proj", "ffn_up": "mlp.up_proj",
                "ffn_down": "mlp.down_proj"}
_BLOCK_RE = re.compile(r"^blk\.(\d+)\.([a-z_]+)\.(weight|bias)$")


def canonical_name(gguf_name: str) -> str:
    if gguf_name in _TOP_NAMES:
        return _TOP_NAMES[gguf_name]
    m = _BLOCK_RE.match(gguf_name)
    if m and m.group(2) in _BLOCK_NAMES:
        return f"model.layers.{int(m.group(1))}.{_BLOCK_NAMES[m.group(2)]}.{m.group(3)}"
    return gguf_name


# ---------------------------------------------------------------------------
# writer (tests, tooling): version 3, little-endian
# ---------------------------------------------------------------------------
def _vtype_of(v: Any) -> int:
    if isinstance(v, bool):
        return VT_BOOL
    if isinstance(v, int):
        return VT_INT64 if v < 0 else VT_UINT64 if v >= 2 ** 32 else VT_UINT32
    if isinstance(v, float):
        return VT_FLOAT32
    if isinstance(v, str):
        return VT_STRING
    if isinstance(v, (list, tuple)):
        return VT_ARRAY
    raise TypeError(f"cannot store {type(v).__name__} in GGUF metadata")


def _pack_string(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _pack_value(v: Any, vtype: int) -> bytes:
    if vtype == VT_STRING:
        return _pack_string(v)
    if vtype == VT_ARRAY:
        et = _vtype_of(v[0]) if len(v) else VT_UINT32
        if et == VT_ARRAY:
            raise TypeError("nested metadata arrays are not written")
        if et in (VT_UINT32, VT_UINT64, VT_INT64) and any(isinstance(x, int) and x < 0 for x in v):
            et = VT_INT64
        return struct.pack("<IQ", et, len(v)) + b"".join(_pack_value(x, et) for x in v)
    return struct.pack(_SCALAR_FMT[vtype], v)


def write_gguf(path: str, tensors: Sequence[Tuple[str, int, Sequence[int], bytes]],
               metadata: Optional[Mapping[str, Any]] = None, alignment: int = DEFAULT_ALIGNMENT) -> None:
    """Write a GGUF v3 file.  `tensors`: (name, ggml_type, row-major shape,
    payload bytes) in file order; metadata values are typed from Python
    (int -> u32/u64/i64, float -> f32, bool, str, list -> array)."""
    meta = dict(metadata or {})
    if alignment != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = alignment
    head = bytearray(GGUF_MAGIC + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for k, v in meta.items():
        vt = VT_UINT32 if k == "general.alignment" else _vtype_of(v)
        head += _pack_string(k) + struct.pack("<I", vt) + _pack_value(v, vt)
    offsets, rel = [], 0
    for name, ttype, shape, payload in tensors:
        need = tensor_nbytes(ttype, shape)
        if len(payload) != need:
            raise DracoFormatError(f"tensor '{name}': payload of {len(payload)} bytes, {need} expected")
        offsets.append(rel)
        rel = -(-(rel + need) // alignment) * alignment
    for (name, ttype, shape, _), off in zip(tensors, offsets):
        dims = list(reversed([int(d) for d in shape]))
        head += _pack_string(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        head += struct.pack("<IQ", ttype, off)
    data_start = -(-len(head) // alignment) * alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data_start - len(head)))
        pos = 0
        for (name, ttype, shape, payload), off in zip(tensors, offsets):
            f.write(b"\0" * (off - pos))
            f.write(bytes(payload))
            pos = off + len(payload)
