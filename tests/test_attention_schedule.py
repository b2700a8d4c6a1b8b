"""Host-side arithmetic of the streaming attention schedule (attention.cu,
attention_stream_kernel), restated and checked on the CPU, plus the workspace
size the C ABI reports for both schedules.

The schedule concatenates the 64-position tiles of all (row group, KV head)
pairs -- pair (g, h) owns tiles [Q[g] + h nt(g), Q[g] + (h + 1) nt(g)) with
nt(g) = ceil(longest context of the group / 64) and Q the prefix over groups
times Hkv -- and CTA c streams the run [W c / G, W (c + 1) / G) over
G = min(grid, W) CTAs. A pair inside one run is written by that CTA; a pair cut
by run boundaries is written by the last of its pieces (a ticket), which reads
the pieces' (acc, m, l) from slot 0 of a CTA whose run starts inside the pair
and from slot 1 of the CTA whose run starts before it. Checked here: every
tile is streamed exactly once; a cut pair's pieces are the consecutive CTAs
run_of(first tile) .. run_of(last tile); no CTA writes two pieces into the
same slot; the combiner's slot rule names the slot each piece was written to.
"""

import numpy as np
import pytest

T = 64


def tiles_per_group(positions, qr):
    rows = len(positions)
    groups = (rows + qr - 1) // qr
    nt = []
    for g in range(groups):
        ends = [p + 1 for p in positions[g * qr:(g + 1) * qr] if p >= 0]
        nt.append((max(ends) + T - 1) // T if ends else 0)
    return nt


def run_begin(w, grid, c):
    return w * c // grid


def run_of(w, grid, i):
    return ((i + 1) * grid + w - 1) // w - 1


def pairs_of(nt, hkv):
    """(pair_start, tiles) for every pair with tiles, in tile-space order."""
    out, start = [], 0
    for n in nt:
        for _ in range(hkv):
            if n:
                out.append((start, n))
            start += n
    return out, start


@pytest.mark.parametrize("seed", range(40))
def test_streaming_runs_cover_every_tile_once_and_cut_pairs_merge_consistently(seed):
    rng = np.random.default_rng(seed)
    rows = int(rng.integers(1, 300))
    hkv = int(rng.choice([1, 2, 4, 8]))
    qr = int(rng.choice([1, 2, 4, 8, 16]))
    positions = rng.integers(0, int(rng.choice([40, 700, 9000])), rows)
    positions[rng.random(rows) < 0.05] = -1  # rows out of range have no tiles
    nt = tiles_per_group(list(positions), qr)
    pairs, w = pairs_of(nt, hkv)
    if w == 0:
        return
    grid = min(int(rng.choice([1, 7, 148, 296, 444, 640])), w)
    cover = np.zeros(w, np.int32)
    slots = {}
    for c in range(grid):
        a, b = run_begin(w, grid, c), run_begin(w, grid, c + 1)
        assert b > a, "every run is non-empty when grid <= W"
        cover[a:b] += 1
        # the run's segments, pair by pair
        for start, n in pairs:
            lo, hi = max(a, start), min(b, start + n)
            if lo >= hi:
                continue
            whole = lo == start and hi == start + n
            if not whole:
                slot = 0 if lo == a else 1  # the kernel: seg_first == run_a
                assert (c, slot) not in slots, "two cut pieces in one slot"
                slots[(c, slot)] = start
    assert np.all(cover == 1)
    for start, n in pairs:
        c_first, c_last = run_of(w, grid, start), run_of(w, grid, start + n - 1)
        assert run_begin(w, grid, c_first) <= start < run_begin(w, grid, c_first + 1)
        if c_first == c_last:
            continue
        for c in range(c_first, c_last + 1):
            sl = 0 if run_begin(w, grid, c) >= start else 1  # the combiner's rule
            assert slots.get((c, sl)) == start


@pytest.mark.parametrize("rows,hq,hkv,d,splits", [(64, 32, 8, 128, 8), (1, 32, 8, 128, 1), (3, 8, 2, 64, 4),
                                                  (256, 32, 8, 128, 64), (5, 16, 16, 64, 2)])
def test_workspace_holds_either_schedule(rows, hq, hkv, d, splits):
    import tmc_cuda
    g = hq // hkv
    split = rows * hq * splits * (d + 2) * 4
    stream = 640 * 2 * g * (d + 2) * 4  # two slots per resident CTA, at most 640 CTAs
    assert tmc_cuda.attention_workspace_bytes(rows, hq, hkv, d, splits) == max(split, stream)
