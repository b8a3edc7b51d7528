"""Seeded random-init checkpoints with the Qwen2.5-0.5B tensor inventory.

The reference's parity fixtures need the real Qwen weights, which are not available, so every
parity and benchmark run uses seeded random-init weights instead: every 2-D weight and every
bias is normal(0, 0.02) in float32, norm gains are 1.  Each tensor draws from its own numpy
PCG64 stream keyed by (seed, index of the tensor in `inventory()`), so a tensor is reproducible
on its own and the order of generation does not matter.

The inventory is the one in the reference's tools/gen_synthetic_safetensors.mjs:13-28: tied
embedding, per layer q/k/v (with biases), o, gate, up, down and two RMSNorm gains, and a final
norm.  Quantisation is then the reference's: int4 everywhere, int8 for the tied embedding
(`tools/quantize.py --embed-dtype q8`).
"""

from __future__ import annotations

import json
import struct
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Dict, Iterator, List, Tuple

import numpy as np

from .format import EMBEDDING, EnargeiaFile, quantize_tensor, write_enargeia


@dataclass(frozen=True)
class ModelConfig:
    """`ModelConfig` of src/model/graph.ts:57-67."""

    layers: int = 24
    hidden: int = 896
    heads: int = 14
    kv_heads: int = 2
    head_dim: int = 64
    intermediate: int = 4864
    vocab: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


QWEN2_0_5B = ModelConfig()
#: A small model with the same structure, for parity runs the CPU oracle finishes in seconds.
TINY = ModelConfig(layers=2, hidden=128, heads=4, kv_heads=2, head_dim=32, intermediate=256, vocab=1000)
#: Mid-size: real head geometry (14/2 x 64, GQA group 7) at 4 layers and a 16k vocabulary.
SMALL = ModelConfig(layers=4, hidden=896, heads=14, kv_heads=2, head_dim=64, intermediate=4864, vocab=16384)


def inventory(cfg: ModelConfig) -> List[Tuple[str, Tuple[int, ...]]]:
    kv = cfg.kv_dim
    specs: List[Tuple[str, Tuple[int, ...]]] = [(EMBEDDING, (cfg.vocab, cfg.hidden))]
    for l in range(cfg.layers):
        p = f"model.layers.{l}"
        specs += [
            (f"{p}.input_layernorm.weight", (cfg.hidden,)),
            (f"{p}.self_attn.k_proj.bias", (kv,)),
            (f"{p}.self_attn.k_proj.weight", (kv, cfg.hidden)),
            (f"{p}.self_attn.o_proj.weight", (cfg.hidden, cfg.hidden)),
            (f"{p}.self_attn.q_proj.bias", (cfg.hidden,)),
            (f"{p}.self_attn.q_proj.weight", (cfg.hidden, cfg.hidden)),
            (f"{p}.self_attn.v_proj.bias", (kv,)),
            (f"{p}.self_attn.v_proj.weight", (kv, cfg.hidden)),
            (f"{p}.post_attention_layernorm.weight", (cfg.hidden,)),
            (f"{p}.mlp.down_proj.weight", (cfg.hidden, cfg.intermediate)),
            (f"{p}.mlp.gate_proj.weight", (cfg.intermediate, cfg.hidden)),
            (f"{p}.mlp.up_proj.weight", (cfg.intermediate, cfg.hidden)),
        ]
    specs.append(("model.norm.weight", (cfg.hidden,)))
    return specs


def random_tensor(seed: int, index: int, name: str, shape: Tuple[int, ...], std: float = 0.02) -> np.ndarray:
    if name.endswith("norm.weight"):
        return np.ones(shape, dtype=np.float32)
    rng = np.random.Generator(np.random.PCG64([seed, index]))
    out = rng.standard_normal(size=shape, dtype=np.float32)
    out *= np.float32(std)
    return out


def random_weights(cfg: ModelConfig, seed: int) -> Iterator[Tuple[str, np.ndarray]]:
    for i, (name, shape) in enumerate(inventory(cfg)):
        yield name, random_tensor(seed, i, name, shape)


def write_safetensors(path: Path, tensors: Dict[str, np.ndarray]) -> None:
    """Minimal F32 safetensors writer (the reference quantiser's input format)."""
    header = {}
    off = 0
    for name in tensors:
        n = tensors[name].size * 4
        header[name] = {"dtype": "F32", "shape": list(tensors[name].shape), "data_offsets": [off, off + n]}
        off += n
    hj = json.dumps(header, separators=(",", ":")).encode()
    with Path(path).open("wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for name in tensors:
            f.write(np.ascontiguousarray(tensors[name], dtype=np.float32).tobytes())


def quantize_weights(cfg: ModelConfig, seed: int, embed_bits: int = 8) -> Iterator[Tuple[str, object]]:
    """Random weights quantised the way `quantize.py --embed-dtype q8` quantises a checkpoint."""
    for name, arr in random_weights(cfg, seed):
        if arr.ndim == 2 and arr.shape[1] % 64 == 0:
            yield name, quantize_tensor(name, arr, embed_bits if name == EMBEDDING else 4)
        else:
            yield name, arr


def build_model_file(cfg: ModelConfig, seed: int, path: Path, embed_bits: int = 8) -> Path:
    """Write the quantised random-init model to `path` (a `.enargeia`) unless it already exists."""
    path = Path(path)
    meta = path.with_suffix(path.suffix + ".json")
    want = {"config": asdict(cfg), "seed": seed, "embed_bits": embed_bits, "format": 1}
    if path.exists() and meta.exists():
        try:
            if json.loads(meta.read_text()) == want:
                return path
        except ValueError:
            pass
    tmp = path.with_suffix(path.suffix + ".tmp")
    write_enargeia(tmp, quantize_weights(cfg, seed, embed_bits))
    tmp.replace(path)
    meta.write_text(json.dumps(want))
    return path


def model_bytes_per_token(f: EnargeiaFile) -> int:
    """Weight bytes one batch-1 decode step must read: every tensor once (the head is tied, so
    the embedding row gather is not counted separately)."""
    return sum(t.nbytes for t in f.tensors.values())
