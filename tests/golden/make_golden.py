"""Regenerate the golden `.enargeia` fixtures with the REFERENCE's own quantiser.

Run in a container where the reference checkout is present (it is read-only; nothing is
written there):

    python tests/golden/make_golden.py --reference /path/to/enargeia

For each case it writes an F32 safetensors into a temporary directory, runs the reference's
`tools/quantize.py` on it unchanged, and copies the `.enargeia` it produced here, together with
`manifest.json` (sha256 of every input tensor and of every output file).  The tests then check
that this package's quantiser and loader reproduce those bytes without the reference present.

Cases:
  tiny_q8   the TINY random-init model (2 layers, hidden 128, vocab 1000), --embed-dtype q8
  tiny_q4   the same weights, --embed-dtype q4 (int4 tied head)
  edges     hand-built blocks: constant, zero, negative constant, endpoints, a large outlier,
            values on exact rounding ties, for both int4 and (via the embedding) int8
"""

from __future__ import annotations

import argparse
import hashlib
import json
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from enargeia_b200.checkpoint import TINY, random_weights, write_safetensors  # noqa: E402

SEED = 1234


def edge_tensors() -> dict:
    """Blocks that exercise every branch of the quantiser."""
    rng = np.random.Generator(np.random.PCG64(99))
    w = rng.standard_normal((8, 128), dtype=np.float32) * np.float32(0.02)
    w[0, :64] = 0.375                      # constant block (scale = |c| / 15)
    w[0, 64:] = 0.0                        # all-zero block (scale = 1)
    w[1, :64] = -0.5                       # negative constant
    w[2, 3] = -1.25                        # endpoints land on codes 0 and 15
    w[2, 40] = 2.5
    w[3, 64:] = np.linspace(-1.0, 1.0, 64, dtype=np.float32)
    w[4, :] *= 0.01
    w[4, 0] = 100.0                        # outlier in one block only
    w[5, :64] = np.arange(64, dtype=np.float32) / np.float32(4.0)  # exact quarter steps: ties
    w[6, 64:] = np.float32(1e-30)          # tiny constant
    # embedding (int8): same tricks at 8 bits
    e = rng.standard_normal((16, 64), dtype=np.float32) * np.float32(0.02)
    e[0, :] = 0.375
    e[1, :] = 0.0
    e[2, :] = -3.0
    e[3, :] = np.arange(64, dtype=np.float32) / np.float32(2.0)
    return {
        "model.embed_tokens.weight": e,
        "model.layers.0.mlp.up_proj.weight": w,
        "model.layers.0.input_layernorm.weight": np.ones(64, dtype=np.float32),
        "model.layers.0.self_attn.q_proj.bias": rng.standard_normal(64, dtype=np.float32),
    }


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="reference checkout (read-only)")
    args = ap.parse_args()
    tool = args.reference / "tools" / "quantize.py"
    if not tool.exists():
        raise SystemExit(f"missing {tool}")

    cases = {
        "tiny_q8": (dict(random_weights(TINY, SEED)), "q8"),
        "tiny_q4": (dict(random_weights(TINY, SEED)), "q4"),
        "edges": (edge_tensors(), "q8"),
    }
    manifest = {"seed": SEED, "tool": "tools/quantize.py (reference, unmodified)", "cases": {}}
    with tempfile.TemporaryDirectory() as tmp:
        for name, (tensors, embed) in cases.items():
            st = Path(tmp) / f"{name}.safetensors"
            out = Path(tmp) / f"{name}.enargeia"
            write_safetensors(st, tensors)
            subprocess.run([sys.executable, str(tool), "--input", str(st), "--output", str(out),
                            "--embed-dtype", embed], check=True, capture_output=True)
            shutil.copy(out, HERE / f"{name}.enargeia")
            manifest["cases"][name] = {
                "embed_dtype": embed,
                "inputs": {k: sha(np.ascontiguousarray(v, dtype=np.float32).tobytes()) for k, v in tensors.items()},
                "output_sha256": sha(out.read_bytes()),
                "output_bytes": out.stat().st_size,
            }
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))
    print(json.dumps({k: v["output_bytes"] for k, v in manifest["cases"].items()}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
