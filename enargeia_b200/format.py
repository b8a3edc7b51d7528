"""The `.enargeia` container and its block quantiser.

The container is the reference's shipping weight format, produced by its `tools/quantize.py`
and parsed by `src/model/enargeia.ts:112-240`:

    "ENARGEIA" | u32 version (1) | u32 header length | JSON header | zero pad to 256 | blob

Every tensor range in the blob starts on a 256-byte boundary.  A quantised tensor (Q4 or Q8)
owns three ranges: `packed` (u32 words, 8 nibbles or 4 bytes each, reduction axis contiguous,
low bits first), `scales` (f32, one per block of 64 along the reduction axis) and `zeros`
(u32 words of packed 4- or 8-bit zero-points).  1-D tensors stay F32.

The quantiser below restates the reference's `quantize_blocks_n` (tools/quantize.py:74-103):
asymmetric, scale = (max - min) / levels in float32, zero = clip(rint(-min / scale)), codes =
clip(rint(v / scale + zero)).  It must produce the reference's bytes exactly; the golden
fixtures under tests/golden/ were written by the reference tool itself and pin it.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, Iterable, Tuple

import numpy as np

MAGIC = b"ENARGEIA"
VERSION = 1
BLOCK = 64
ALIGN = 256
EMBEDDING = "model.embed_tokens.weight"


class EnargeiaError(ValueError):
    """A malformed or unsupported `.enargeia` file (src/model/enargeia.ts:68-74)."""


@dataclass
class QuantTensor:
    """One block-quantised tensor, the `QuantTensor` of src/model/weights.ts:56-67."""

    name: str
    bits: int  # 4 or 8
    shape: Tuple[int, int]  # (rows = output features, cols = reduction axis)
    packed: np.ndarray  # u32
    scales: np.ndarray  # f32
    zeros: np.ndarray  # u32
    block_size: int = BLOCK

    @property
    def rows(self) -> int:
        return self.shape[0]

    @property
    def cols(self) -> int:
        return self.shape[1]

    @property
    def blocks_per_row(self) -> int:
        return self.cols // self.block_size

    @property
    def nbytes(self) -> int:
        return self.packed.nbytes + self.scales.nbytes + self.zeros.nbytes

    def dequantize(self) -> np.ndarray:
        """(q - zero) * scale as float32, exactly the shader's per-element dequantisation."""
        per = 32 // self.bits
        mask = (1 << self.bits) - 1
        shifts = np.arange(per, dtype=np.uint32) * self.bits
        q = ((self.packed[:, None] >> shifts) & mask).reshape(-1)
        nblocks = self.rows * self.blocks_per_row
        z = ((self.zeros[:, None] >> shifts) & mask).reshape(-1)[:nblocks]
        out = (q.reshape(nblocks, self.block_size).astype(np.float32) - z[:, None].astype(np.float32))
        out *= self.scales[:, None]
        return out.reshape(self.rows, self.cols)


@dataclass
class F32Tensor:
    name: str
    shape: Tuple[int, ...]
    data: np.ndarray

    @property
    def nbytes(self) -> int:
        return self.data.nbytes


@dataclass
class EnargeiaFile:
    tensors: Dict[str, object] = field(default_factory=dict)
    header: dict = field(default_factory=dict)

    def quant(self, name: str) -> QuantTensor:
        t = self.tensors[name]
        if not isinstance(t, QuantTensor):
            raise EnargeiaError(f"{name} is not a quantised tensor")
        return t

    def f32(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        if not isinstance(t, F32Tensor):
            raise EnargeiaError(f"{name} is not an F32 tensor")
        return t.data


# ---------------------------------------------------------------------------------------------
# quantisation


def quantize_blocks(values: np.ndarray, bits: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Asymmetric `bits`-bit quantisation in blocks of 64 along the last axis.

    Returns (packed u32, scales f32, zeros u32).  Same float32 arithmetic, rounding (rint: half
    to even) and packing order as tools/quantize.py:74-103, so the bytes are identical.
    """
    levels = np.float32((1 << bits) - 1)
    per_word = 32 // bits
    rows, cols = values.shape
    if cols % BLOCK:
        raise EnargeiaError(f"reduction axis {cols} is not a multiple of {BLOCK}")
    blocks = np.ascontiguousarray(values, dtype=np.float32).reshape(rows * cols // BLOCK, BLOCK)

    lo = blocks.min(axis=1)
    hi = blocks.max(axis=1)
    scale = (hi - lo) / levels
    degenerate = scale <= 0
    if degenerate.any():
        # A constant block: |c|/levels puts the constant on the top (or bottom) code; an
        # all-zero block gets scale 1.
        alt = np.where(hi != 0, np.abs(hi) / levels, np.float32(1.0)).astype(np.float32)
        scale = np.where(degenerate, alt, scale).astype(np.float32)
    zero = np.clip(np.rint(-lo / scale), 0, levels).astype(np.int64)

    # quantize.py adds the int64 zero-point to the float32 quotient, which numpy promotes to
    # float64 before rint: the same promotion is kept here (in chunks, to bound memory).
    q = np.empty(blocks.shape, dtype=np.uint32)
    step = 1 << 18
    for b in range(0, blocks.shape[0], step):
        e = min(b + step, blocks.shape[0])
        t = (blocks[b:e] / scale[b:e, None]).astype(np.float64)
        t += zero[b:e, None]
        np.rint(t, out=t)
        np.clip(t, 0, float(levels), out=t)
        q[b:e] = t.astype(np.uint32)

    shifts = np.arange(per_word, dtype=np.uint32) * np.uint32(bits)
    qw = q.reshape(-1, per_word)
    packed = np.zeros(qw.shape[0], dtype=np.uint32)
    for j in range(per_word):
        packed |= qw[:, j] << shifts[j]

    n_blocks = zero.shape[0]
    padded = np.zeros(((n_blocks + per_word - 1) // per_word) * per_word, dtype=np.uint32)
    padded[:n_blocks] = zero.astype(np.uint32)
    pw = padded.reshape(-1, per_word)
    zeros_packed = np.zeros(pw.shape[0], dtype=np.uint32)
    for j in range(per_word):
        zeros_packed |= pw[:, j] << shifts[j]
    return packed, scale.astype(np.float32), zeros_packed


def quantize_tensor(name: str, matrix: np.ndarray, bits: int) -> QuantTensor:
    packed, scales, zeros = quantize_blocks(matrix, bits)
    return QuantTensor(name, bits, (int(matrix.shape[0]), int(matrix.shape[1])), packed, scales, zeros)


# ---------------------------------------------------------------------------------------------
# writing


def write_enargeia(path: Path, tensors: Iterable[Tuple[str, object]], generator: str = "tools/quantize.py") -> int:
    """Write tensors (already quantised, or F32) in sorted-name order, as quantize.py does.

    Returns the file size.  `tensors` yields (name, QuantTensor | np.ndarray).
    """
    entries: Dict[str, dict] = {}
    chunks = []
    cursor = 0

    def append(payload: bytes):
        nonlocal cursor
        pad = (-cursor) % ALIGN
        if pad:
            chunks.append(b"\0" * pad)
            cursor += pad
        begin = cursor
        chunks.append(payload)
        cursor += len(payload)
        return [begin, cursor]

    for name, t in sorted(tensors, key=lambda kv: kv[0]):
        if isinstance(t, QuantTensor):
            entries[name] = {
                "dtype": "Q4" if t.bits == 4 else "Q8",
                "shape": [t.rows, t.cols],
                "blockSize": BLOCK,
                "offsets": {
                    "packed": append(t.packed.tobytes()),
                    "scales": append(t.scales.tobytes()),
                    "zeros": append(t.zeros.tobytes()),
                },
            }
        else:
            arr = np.asarray(t, dtype=np.float32)
            entries[name] = {
                "dtype": "F32",
                "shape": list(arr.shape),
                "offsets": {"data": append(arr.tobytes())},
            }
    header_json = json.dumps(
        {
            "generator": generator,
            "blockSize": BLOCK,
            "quantization": "asymmetric-int4-blockwise",
            "tensors": entries,
        },
        separators=(",", ":"),
    ).encode("utf-8")
    prefix_len = len(MAGIC) + 8 + len(header_json)
    pad = (-prefix_len) % ALIGN
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("wb") as handle:
        handle.write(MAGIC)
        handle.write(struct.pack("<I", VERSION))
        handle.write(struct.pack("<I", len(header_json)))
        handle.write(header_json)
        handle.write(b"\0" * pad)
        for c in chunks:
            handle.write(c)
    return path.stat().st_size


# ---------------------------------------------------------------------------------------------
# reading


def read_enargeia(path: Path) -> EnargeiaFile:
    """Parse a `.enargeia` file into numpy views (a read-only memory map of the blob)."""
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    return parse_enargeia(raw)


def parse_enargeia(raw: np.ndarray) -> EnargeiaFile:
    if raw.shape[0] < 16:
        raise EnargeiaError("need at least 16 bytes to read the header length")
    if bytes(raw[:8]) != MAGIC:
        raise EnargeiaError(f"not a .enargeia file: magic is {bytes(raw[:8])!r}")
    version, header_len = struct.unpack("<II", bytes(raw[8:16]))
    if version != VERSION:
        raise EnargeiaError(f"unsupported .enargeia version {version}, expected {VERSION}")
    if 16 + header_len > raw.shape[0]:
        raise EnargeiaError("header runs past the end of the file")
    header = json.loads(bytes(raw[16 : 16 + header_len]).decode("utf-8"))
    data_offset = 16 + header_len
    data_offset += (-data_offset) % ALIGN
    out = EnargeiaFile(header=header)

    def view(rng, dtype):
        b, e = rng
        if b % ALIGN or e < b or data_offset + e > raw.shape[0]:
            raise EnargeiaError(f"bad byte range {rng}")
        return raw[data_offset + b : data_offset + e].view(dtype)

    for name, entry in header["tensors"].items():
        dt = entry["dtype"]
        shape = tuple(int(s) for s in entry["shape"])
        offs = entry["offsets"]
        if dt in ("Q4", "Q8"):
            bits = 4 if dt == "Q4" else 8
            block = int(entry.get("blockSize", BLOCK))
            if block != BLOCK:
                raise EnargeiaError(f"{name}: block size {block} unsupported")
            t = QuantTensor(name, bits, (shape[0], shape[1]), view(offs["packed"], np.uint32),
                            view(offs["scales"], np.float32), view(offs["zeros"], np.uint32), block)
            per = 32 // bits
            nb = shape[0] * shape[1] // block
            if (t.packed.shape[0] != shape[0] * shape[1] // per or t.scales.shape[0] != nb
                    or t.zeros.shape[0] != (nb + per - 1) // per):
                raise EnargeiaError(f"{name}: range sizes do not match shape {shape}")
            out.tensors[name] = t
        elif dt == "F32":
            out.tensors[name] = F32Tensor(name, shape, view(offs["data"], np.float32).reshape(shape))
        else:
            raise EnargeiaError(f"{name}: dtype {dt} unsupported on this path")
    return out
