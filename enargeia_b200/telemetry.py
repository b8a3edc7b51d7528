"""Per-kernel-group shares of a decode step, in the groups of src/runtime/telemetry.ts:12-20.

The reference colours each WGSL dispatch by a name pattern (embedding, rmsnorm, projection, rope,
attention, mlp, sample) and reports each group's share of the step (BENCH.md's share table).
Here a step is two weight-streaming kernels and the sampler, so the shares come from two sources:

- the persistent layer kernel's stage trace (enx_trace, one traced CTA): inside every layer it
  stamps the norm, the q|k|v rows (projection; RoPE and the f16 cache pack are fused into their
  epilogue), attention, the o rows, gate|up and down; the time a stage spends waiting for the
  previous stage's tagged outputs is its own row, "handoff" (WebGPU pays the same thing as
  dispatch boundaries, which its profiler does not show);
- CUDA-event times of the tied-head kernel (group "embedding": lm_head) and of the sampler.
"""

from __future__ import annotations

from typing import Dict

import numpy as np

GROUPS = ["embedding", "rmsnorm", "projection", "rope", "attention", "mlp", "sample", "handoff"]

DETAIL = 14  # detail stamps per layer (k_mega.cuh kMegaTraceDetail)


def trace_words(layers: int) -> int:
    """Length of the stage trace enx_trace fills: 3 stamps per stage (3 stages a layer, plus the
    end), then DETAIL stamps per layer, then two spare words."""
    return 3 * (3 * layers + 1) + DETAIL * layers + 2


def parse_stage_trace(buf, layers: int) -> Dict[str, float]:
    """Stage intervals (us, summed over layers) from the traced CTA's %globaltimer stamps.

    Per layer the persistent kernel stamps each stage's start, the moment its weights are
    resident and its end (A: q|k|v units, attention and o rows; C: gate|up; D: down), and inside
    the stages: A after the x read (7), after the norm (0), after the units (1), after the q|k|v
    handoff (2), after the q and current k|v loads (3), after attention (4), after the attention
    outputs are in (5); C after the norm (11) and after the dot products (12); D after the gated
    read (13)."""
    L = layers
    t = np.asarray(buf[: 3 * (3 * L + 1)], dtype=np.float64).reshape(-1, 3) / 1e3
    d = np.asarray(buf[3 * (3 * L + 1): 3 * (3 * L + 1) + DETAIL * L], dtype=np.float64).reshape(L, DETAIL) / 1e3
    names = ["attn", "gate_up", "down"]
    out = {f"{k}_{p}": 0.0 for k in names for p in ("wait", "weights", "compute")}
    for i in range(3 * L):
        k = names[i % 3]
        prev_done = t[i - 1, 2] if i > 0 else t[i, 0]
        out[f"{k}_wait"] += t[i, 0] - prev_done          # after the previous stage
        out[f"{k}_weights"] += max(t[i, 1] - t[i, 0], 0.0)  # slot wait (C: x_mid read + slot wait)
        out[f"{k}_compute"] += t[i, 2] - t[i, 1]
    out["total"] = t[3 * L, 2] - t[0, 0]
    if d.any():
        A0, A1, A2 = t[0:3 * L:3, 0], t[0:3 * L:3, 1], t[0:3 * L:3, 2]
        C1, C2 = t[1:3 * L:3, 1], t[1:3 * L:3, 2]
        D0, D1 = t[2:3 * L:3, 0], t[2:3 * L:3, 1]
        seq = np.concatenate([A0[:, None], d[:, :6], A2[:, None]], axis=1)
        for j, m in enumerate(["norm", "units", "ready_wait", "q_load", "attention", "done_wait", "o_rows+end"]):
            out[f"attn.{m}"] = float(np.sum(seq[:, j + 1] - seq[:, j]))
        out["attn.x_read"] = float(np.sum(d[:, 7] - A1))        # layer 0: the embedding rows
        out["attn.norm_compute"] = float(np.sum(d[:, 0] - d[:, 7]))
        out["gate_up.norm"] = float(np.sum(d[:, 11] - C1))
        out["gate_up.dots"] = float(np.sum(d[:, 12] - d[:, 11]))
        out["gate_up.silu"] = float(np.sum(C2 - d[:, 12]))
        out["down.read"] = float(np.sum(d[:, 13] - D0))
        out["down.prep"] = float(np.sum(D1 - d[:, 13]))        # chunk sums + slot wait
    return out


def layer_groups(stage: Dict[str, float]) -> Dict[str, float]:
    """Microseconds per group over all layers, from Model.stage_times() of a traced step."""
    g = {k: 0.0 for k in GROUPS}
    get = stage.get
    g["attention"] += get("attn.q_load", 0.0) + get("attn.attention", 0.0)
    g["handoff"] += get("attn_wait", 0.0) + get("attn.ready_wait", 0.0) + get("attn.done_wait", 0.0)
    g["handoff"] += get("gate_up_wait", 0.0) + get("gate_up_weights", 0.0) + get("down_wait", 0.0)
    g["projection"] += get("attn.units", 0.0) + get("attn.o_rows+end", 0.0) + get("down_compute", 0.0)
    if "gate_up.dots" in stage:
        # stage A's start: slot wait + x read (handoff), then the norm itself; C: norm, dot
        # products, SiLU; D: the gated read (handoff), then chunk sums + slot wait
        g["handoff"] += get("attn.norm", 0.0) - get("attn.norm_compute", 0.0) + get("down.read", 0.0)
        g["rmsnorm"] += get("attn.norm_compute", 0.0) + get("gate_up.norm", 0.0)
        g["projection"] += get("gate_up.dots", 0.0) + get("down.prep", 0.0)
        g["mlp"] += get("gate_up.silu", 0.0)
    else:
        g["rmsnorm"] += get("attn.norm", 0.0)
        g["projection"] += get("gate_up_compute", 0.0)
        g["handoff"] += get("down_weights", 0.0)
    return g


def step_shares(stage: Dict[str, float], head_us: float, sample_us: float, step_us: float) -> Dict[str, Dict[str, float]]:
    """The share table: per group, microseconds and share of the measured step."""
    g = layer_groups(stage)
    g["embedding"] += head_us
    g["sample"] += sample_us
    accounted = sum(g.values())
    g["other"] = max(step_us - accounted, 0.0)  # prep kernel, launch gaps, untraced remainder
    return {k: {"us": round(v, 2), "share": round(v / step_us, 4) if step_us else 0.0} for k, v in g.items()}
