"""K-tile flags of observation rows (the words the fused step writes and the
MLP policy reads to skip all-zero first-layer K tiles): the host helpers
against a plain restatement of the layout -- tile t covers row entries
[64 t, 64 t + 64) and is bit min(t >> 2, 31) of word t & 3."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from qqt_b200.sim import check_tile_flags, tile_flag_words, tile_flags


def _words_loop(row: np.ndarray) -> list[int]:
    words = [0, 0, 0, 0]
    bits = row.view(np.uint16)
    for t in range((row.size + 63) // 64):
        if bits[64 * t: 64 * t + 64].any():
            words[t & 3] |= 1 << min(t >> 2, 31)
    return [w - (1 << 32) if w >= 1 << 31 else w for w in words]


@pytest.mark.parametrize("k", [2368, 2366, 64 * 140 + 8])
def test_tile_flags_match_layout(k):
    rng = np.random.default_rng(k)
    n = 24
    rows = np.zeros((n, k), np.float16)
    for i in range(n):
        cols = rng.choice(k, size=rng.integers(0, 12), replace=False)
        rows[i, cols] = rng.choice([1.0, -0.0, 0.25, -3.0], size=cols.size)
    got = tile_flags(torch.from_numpy(rows)).numpy()
    want = np.array([_words_loop(r) for r in rows], np.int64).astype(np.int32)
    assert np.array_equal(got, want)


def test_range_words_equal_flags_of_a_filled_range():
    k = 2368
    for lo, hi in [(0, 1), (1183, 1352), (63, 65), (2300, 2368)]:
        row = torch.zeros((1, k), dtype=torch.float16)
        row[0, lo:hi] = 1
        assert torch.equal(tile_flags(row)[0], tile_flag_words(lo, hi, "cpu"))


def test_flag_tensor_checks():
    check_tile_flags(torch.zeros((5, 4), dtype=torch.int32), 5)
    for bad in (torch.zeros((5, 4), dtype=torch.int64), torch.zeros((5, 3), dtype=torch.int32),
                torch.zeros((4, 5), dtype=torch.int32).t()):
        with pytest.raises(ValueError):
            check_tile_flags(bad, 5)
