"""The per-group share table of a decode step (enargeia_b200/telemetry.py), the reference's
telemetry groups (src/runtime/telemetry.ts:12-20: embedding, rmsnorm, projection, rope,
attention, mlp, sample) plus the handoffs between the persistent kernel's stages, built here from
synthetic stage times: every stage lands in exactly one group, the head and sampler times are
added in, and what the trace does not account for is "other"."""

import pytest

from enargeia_b200.telemetry import GROUPS, layer_groups, step_shares

STAGE = {  # us summed over the layers, the keys Model.stage_times() returns
    "attn_wait": 2.0, "attn_weights": 15.0, "attn_compute": 260.0,
    "gate_up_wait": 0.5, "gate_up_weights": 35.0, "gate_up_compute": 100.0,
    "down_wait": 0.8, "down_weights": 85.0, "down_compute": 55.0,
    "attn.norm": 60.0, "attn.units": 23.0, "attn.ready_wait": 21.0, "attn.q_load": 3.0,
    "attn.attention": 65.0, "attn.done_wait": 23.0, "attn.o_rows+end": 49.0,
}


def test_reference_groups_are_all_present():
    assert set(GROUPS) >= {"embedding", "rmsnorm", "projection", "rope", "attention", "mlp", "sample"}
    g = layer_groups(STAGE)
    assert set(g) == set(GROUPS)


def test_every_stage_lands_in_one_group():
    g = layer_groups(STAGE)
    assert g["rmsnorm"] == pytest.approx(60.0)
    assert g["projection"] == pytest.approx(23.0 + 49.0 + 100.0 + 55.0)
    assert g["attention"] == pytest.approx(3.0 + 65.0)
    assert g["handoff"] == pytest.approx(2.0 + 21.0 + 23.0 + 0.5 + 35.0 + 0.8 + 85.0)
    assert g["embedding"] == g["sample"] == 0.0


def test_shares_of_the_measured_step():
    step_us = 600.0
    t = step_shares(STAGE, head_us=33.0, sample_us=9.0, step_us=step_us)
    assert set(t) == set(GROUPS) | {"other"}
    assert t["embedding"]["us"] == pytest.approx(33.0)
    assert t["sample"]["us"] == pytest.approx(9.0)
    accounted = sum(v["us"] for k, v in t.items() if k != "other")
    assert t["other"]["us"] == pytest.approx(step_us - accounted, abs=0.05)
    assert sum(v["share"] for v in t.values()) == pytest.approx(1.0, abs=1e-3)


def test_other_is_never_negative():
    t = step_shares(STAGE, head_us=33.0, sample_us=9.0, step_us=100.0)  # trace longer than the step
    assert t["other"]["us"] == 0.0


def _synthetic_trace(layers):
    """A trace buffer with a known length for every interval of every layer (ns stamps)."""
    import numpy as np

    from enargeia_b200.telemetry import DETAIL, trace_words

    # per layer, in time order: (stamp, length of the interval that ends at it in ns)
    order = [("A0", 100), ("A1", 200), ("d7", 300), ("d0", 400), ("d1", 500), ("d2", 600), ("d3", 700),
             ("d4", 800), ("d5", 900), ("A2", 1000), ("C0", 1100), ("C1", 1200), ("d11", 1300),
             ("d12", 1400), ("C2", 1500), ("D0", 1600), ("d13", 1700), ("D1", 1800), ("D2", 1900)]
    buf = np.zeros(trace_words(layers), dtype=np.uint64)
    base = 3 * (3 * layers + 1)
    now = 1_000_000
    first = None
    for l in range(layers):
        for name, dt in order:
            now += dt
            if first is None:
                first = now
            if name[0] in "ACD" and name[1:].isdigit():
                stage = {"A": 0, "C": 1, "D": 2}[name[0]]
                buf[3 * (3 * l + stage) + int(name[1])] = now
            else:
                buf[base + DETAIL * l + int(name[1:])] = now
    buf[3 * (3 * layers)] = now + 10
    buf[3 * (3 * layers) + 2] = now + 20
    return buf, first, now


def test_parse_stage_trace_and_groups_partition_the_timeline():
    from enargeia_b200.telemetry import parse_stage_trace

    L = 3
    buf, first, last = _synthetic_trace(L)
    st = parse_stage_trace(buf, L)
    us = lambda ns: ns / 1e3  # noqa: E731
    assert st["attn.x_read"] == pytest.approx(us(300) * L)
    assert st["attn.norm_compute"] == pytest.approx(us(400) * L)
    assert st["attn.attention"] == pytest.approx(us(800) * L)
    assert st["gate_up.norm"] == pytest.approx(us(1300) * L)
    assert st["gate_up.dots"] == pytest.approx(us(1400) * L)
    assert st["gate_up.silu"] == pytest.approx(us(1500) * L)
    assert st["down.read"] == pytest.approx(us(1700) * L)
    assert st["down.prep"] == pytest.approx(us(1800) * L)
    g = layer_groups(st)
    assert g["mlp"] == pytest.approx(us(1500) * L)
    assert g["rmsnorm"] == pytest.approx(us(400 + 1300) * L)
    # the groups cover the traced CTA's timeline from its first stamp to the last stage's end
    assert sum(g.values()) == pytest.approx(us(last - first))
