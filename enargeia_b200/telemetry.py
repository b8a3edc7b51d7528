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

GROUPS = ["embedding", "rmsnorm", "projection", "rope", "attention", "mlp", "sample", "handoff"]


def layer_groups(stage: Dict[str, float]) -> Dict[str, float]:
    """Microseconds per group over all layers, from Model.stage_times() of a traced step."""
    g = {k: 0.0 for k in GROUPS}
    g["rmsnorm"] += stage.get("attn.norm", 0.0)
    g["projection"] += stage.get("attn.units", 0.0) + stage.get("attn.o_rows+end", 0.0)
    g["attention"] += stage.get("attn.q_load", 0.0) + stage.get("attn.attention", 0.0)
    g["handoff"] += stage.get("attn_wait", 0.0) + stage.get("attn.ready_wait", 0.0) + stage.get("attn.done_wait", 0.0)
    # gate|up: its "weights" span holds the tagged read of x_mid; compute holds norm + rows + SiLU
    g["handoff"] += stage.get("gate_up_wait", 0.0) + stage.get("gate_up_weights", 0.0)
    g["projection"] += stage.get("gate_up_compute", 0.0)
    g["handoff"] += stage.get("down_wait", 0.0) + stage.get("down_weights", 0.0)
    g["projection"] += stage.get("down_compute", 0.0)
    return g


def step_shares(stage: Dict[str, float], head_us: float, sample_us: float, step_us: float) -> Dict[str, Dict[str, float]]:
    """The share table: per group, microseconds and share of the measured step."""
    g = layer_groups(stage)
    g["embedding"] += head_us
    g["sample"] += sample_us
    accounted = sum(g.values())
    g["other"] = max(step_us - accounted, 0.0)  # prep kernel, launch gaps, untraced remainder
    return {k: {"us": round(v, 2), "share": round(v / step_us, 4) if step_us else 0.0} for k, v in g.items()}
