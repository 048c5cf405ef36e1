"""bench.py's host-side helpers on CPU: the decoder of the MoE kernel's timeline buffer (the encoding documented
with ``dbg`` in include/qwenfast_b200.h)."""
import torch

import bench


def _enc(t_ns, tag, base=1796180000000000000):
    v = ((base + t_ns) << 12 | tag) & ((1 << 64) - 1)
    return v - (1 << 64) if v >= (1 << 63) else v


def test_decode_timeline():
    d = torch.zeros(512, 32, dtype=torch.int64)
    for c in range(3):
        d[c, 31] = _enc(100 * c, 0xFFF)                                   # CTA entries; the earliest is t = 0
        events = [(9000, 30), (10000, 3), (18000 + c, 19), (20000, 6), (24000, 22), (40000 + 1000 * c, 31)]
        for j, (t, code) in enumerate(events):
            d[c, j] = _enc(t, code | (c % 3) << 5)
    d[0, 10] = _enc(12000, 3 | 1 << 5)                                    # a second pipeline of CTA 0, item left open
    out = bench.decode_timeline(d.view(-1), 3)
    assert out["consumers_start_us"] == 9.0 and out["last_stop_us"] == 42.0
    g1, g2 = out["kinds"]["G1"], out["kinds"]["G2"]
    assert g1["n"] == 4 and g1["first_start_us"] == 10.0 and g1["last_start_us"] == 12.0
    assert g1["stages_us_median"] == 8.0 and g1["last_stages_done_us"] == 18.0
    assert g2["n"] == 3 and g2["stages_us_max"] == 4.0 and g2["last_stages_done_us"] == 24.0
