"""The decode-step trace summary of bench.py (`--trace`) on a synthetic
timeline with known phases (no GPU): launches grouped per step in issue
order, a captured launch's tag replayed once per step, the LM head's own
tag per step."""

import numpy as np

import bench


def _launch(tag, base, ctas=3, wait=1000, loop=5000, loop_skew=200, tail=300, head=None):
    rows = []
    for c in range(ctas):
        t0 = base + 100 * c
        t1 = t0 + wait
        t2 = t1 + loop + loop_skew * c
        x0 = x1 = 0
        if head is not None:  # LM head: own top-k end, ticket end
            x0, x1 = t2 + head[0], t2 + head[0] + head[1]
            t3 = x1 + (head[2] if c == ctas - 1 else 0)
        else:
            t3 = t2 + tail
        rows.append([(tag << 32) | c, c, t0, t1, t2, t3, x0, x1])
    return rows


def test_summary_of_a_synthetic_two_step_trace():
    layers, roles = 2, len(bench.TRACE_ROLES)
    rec = []
    for step in range(2):
        base = step * 3_000_000  # steps 3 ms apart
        for j in range(layers * roles):  # captured launches: the same tag every step
            rec += _launch(j, base + j * 10_000)
        rec += _launch(100 + step, base + layers * roles * 10_000, head=(800, 50, 700))
    out = bench.summarize_trace(np.array(rec, dtype=np.int64), layers=layers)

    assert out["steps"] == 2
    qkv = out["roles_us"]["qkv"]
    # every launch is shifted by 10 us from the previous one
    assert qkv["interval"] == 10.0
    # loop: last wait (CTA 2 at +200 + 1000) -> last loop end (CTA 2 at +200 + 1000 + 5000 + 400)
    assert qkv["loop"] == 5.4
    assert qkv["loop_spread"] == 0.6 and qkv["tail"] == 0.3
    # the first wait (CTA 0 at +1000) after the previous launch's last end (-10000 + 6600 + 300)
    assert qkv["wait_release"] == round((10_000 + 1000 - 6900) / 1e3, 2)
    assert out["lm_head_tail_us"] == {"topk": 0.8, "ticket": 0.05, "merge": 0.7}
    head_end = layers * roles * 10_000 + 200 + 1000 + 5400 + 850 + 700
    assert out["step_us"] == [round(head_end / 1e3, 1)] * 2
