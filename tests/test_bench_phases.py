"""The benchmark's phase-stamp analysis (bench.py --phase-stamps) on
synthetic records with known answers: per-launch spans of a kernel (the
k-th record of a block or warp belongs to its k-th launch), per-phase
durations, and the chain summary that says what gates a step's start."""

from __future__ import annotations

import numpy as np

import bench


def _rec(kid, ph, block, warp, t):
    w0 = (kid << 56) | (ph << 48) | (3 << 32) | (block << 8) | warp
    return [w0, t]


def _records():
    """Two ticks of one group: policy (kid 1, CTAs 0-1, stamps 0, 5, 14),
    bot (kid 3, warps of block 0, stamps 0 and 4) and step (kid 2, warps of
    blocks 0-1, stamps 0 and 17); times in ns."""
    r = []
    for k, base in enumerate((0, 60_000)):
        for cta in (0, 1):
            r.append(_rec(1, 0, cta, 0, base + 100 * cta))
            r.append(_rec(1, 5, cta, 0, base + 12_000 + 100 * cta))
            r.append(_rec(1, 14, cta, 0, base + 27_000 + 100 * cta))
        for w in (0, 1):
            r.append(_rec(3, 0, 0, w, base + 2_000 + 50 * w))
            r.append(_rec(3, 4, 0, w, base + 20_000 + 50 * w))
        for blk in (0, 1):
            for w in (0, 1):
                s0 = base + 21_000 + 1_000 * blk          # after the bot has ended
                r.append(_rec(2, 0, blk, w, s0))
                r.append(_rec(2, 17, blk, w, s0 + 29_000 + 10 * w))
    return np.array(r, dtype=np.uint64)


def test_launch_spans_group_records_by_launch():
    rec = _records()
    P = bench.launch_spans(rec, 1, 0, 14, False)
    assert P.tolist() == [[0, 100, 27_100], [60_000, 60_100, 87_100]]
    A = bench.launch_spans(rec, 3, 0, 4, True)
    assert A.tolist() == [[2_000, 2_050, 20_050], [62_000, 62_050, 80_050]]
    S = bench.launch_spans(rec, 2, 0, 17, True)
    assert S.tolist() == [[21_000, 22_000, 51_010], [81_000, 82_000, 111_010]]


def test_phase_table_durations():
    lines = bench.phase_table(_records(), 11)     # policy: stamps 0, 1, ... (absent here)
    assert lines[0].endswith("no records")
    rec = _records()
    # a table over stamps the records hold: policy 0 -> 5 -> 14
    saved = bench.PHASES[11]
    try:
        bench.PHASES[11] = ("policy", [0, 5, 14], ["layer 1", "tail"], False, 1)
        lines = bench.phase_table(rec, 11)
    finally:
        bench.PHASES[11] = saved
    assert "4 samples" in lines[0] and "total mean 27.00 us" in lines[0]
    assert "mean  12.00" in lines[1] and "mean  15.00" in lines[2]


def test_chain_summary_reports_what_gates_the_step():
    lines = bench.chain_summary(_records())
    text = "\n".join(lines)
    # a step starts 21 us after its policy's first CTA: 6.1 us before the
    # policy's last CTA ends (27.1 us), 8.9 us after its layer 1 (12.1 us)
    # and 0.95 us after its bot (20.05 us); it ends 8.99 us before the next
    # policy starts
    assert "step end -> next policy start 8.99 us" in text
    assert "step's first block starts 6.10 us before its policy ends" in text
    assert "step ends 23.91 us after it" in text
    assert "8.90 us after its policy's layer 1 ends and 0.95 us after the latest bot" in text
    assert "a bot launch ends 20.05 us after the policy launch" in text
    assert "bot span 18.05 us" in text
    assert "policy span 27.10 us (CTA start spread 0.10)" in text
