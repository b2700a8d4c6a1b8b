"""Host-side plan of the stream-K tcgen05 GEMM (gemm.cu plan_gemm /
gemm_workspace_floats, exported through tmc_k_batched_gemm_workspace_bytes),
checked on the CPU against a restatement, plus the run / piece arithmetic the
kernel's three roles share (RunCursor, run_of, the closers): every
(tile, K block) iteration is streamed exactly once, a split tile's pieces are
the consecutive runs run_of(first) .. run_of(last), each writes its own
workspace slot, and the closers are the pieces whose runs end inside the tile."""

import pytest

TILE_ROWS, ATOM, MIN_RUN_K, SMS = 128, 64, 256, 148


def k_atoms(tn):
    """64-column swizzle atoms per pipeline stage (gemm.cuh gemm_k_atoms)."""
    return 4 if tn <= 64 else 2 if tn <= 128 else 1


def plan(n, k, m, sms=SMS):
    tn = 16 if m <= 16 else 32 if m <= 32 else 64 if m <= 64 else 128
    block = ATOM * k_atoms(tn)  # K elements per pipeline stage
    tiles, kblocks = (n + TILE_ROWS - 1) // TILE_ROWS, (k + block - 1) // block
    iters = tiles * kblocks
    min_run = (MIN_RUN_K + block - 1) // block
    grid = max(1, min(sms, iters // min_run))
    return tn, tiles, kblocks, grid


def workspace_bytes(n, k, m):
    tn, tiles, kblocks, grid = plan(n, k, m)
    iters = tiles * kblocks
    partial = any(iters * c // grid % kblocks for c in range(1, grid))
    floats = grid * 2 * tn * TILE_ROWS if partial else 0
    return (floats * 4 + 255) // 256 * 256 + tiles * 8


def run_begin(iters, grid, c):
    return iters * c // grid


def run_of(iters, grid, i):
    return ((i + 1) * grid + iters - 1) // iters - 1


SHAPES = [(6144, 4096, 64), (4096, 4096, 64), (28672, 4096, 64), (4096, 14336, 64), (128256, 4096, 64),
          (2816, 1024, 12), (4096, 1408, 33), (1000, 136, 17), (128, 8, 9), (40, 64, 128), (14336, 2048, 100)]
# Per-rank shards of the 8B projections at bs64 under tensor parallelism 2 / 4 / 8:
# QKV and gate/up split their outputs, O and down their inputs, the LM head its vocabulary.
SHAPES += [shape for tp in (2, 4, 8) for shape in
           ((6144 // tp, 4096, 64), (4096, 4096 // tp, 64), (28672 // tp, 4096, 64), (4096, 14336 // tp, 64),
            (128256 // tp, 4096, 64))]


@pytest.mark.parametrize("n,k,m", SHAPES)
def test_workspace_bytes_match_the_plan(n, k, m):
    import tmc_cuda
    assert tmc_cuda.batched_gemm_workspace_bytes(n, k, m) == workspace_bytes(n, k, m)


@pytest.mark.parametrize("n,k,m", SHAPES)
@pytest.mark.parametrize("sms", [SMS, 132, 7, 1])
def test_stream_k_runs_cover_every_iteration_once(n, k, m, sms):
    _, tiles, kblocks, grid = plan(n, k, m, sms)
    iters = tiles * kblocks
    cover = [0] * iters
    pieces = {}
    for c in range(grid):
        nxt, end, idx = run_begin(iters, grid, c), run_begin(iters, grid, c + 1), 0
        assert end > nxt, "every run streams at least one iteration"
        while nxt < end:
            t = nxt // kblocks
            kb0, kb1 = nxt - t * kblocks, min(end - t * kblocks, kblocks)
            for i in range(t * kblocks + kb0, t * kblocks + kb1):
                cover[i] += 1
            if not (kb0 == 0 and kb1 == kblocks):
                pieces.setdefault(t, []).append((c, 0 if idx == 0 else 1, t * kblocks + kb1 <= run_begin(iters, grid, c + 1)
                                                 and run_begin(iters, grid, c + 1) <= (t + 1) * kblocks))
            idx += 1
            nxt = t * kblocks + kb1
    assert all(x == 1 for x in cover)
    slots = set()
    for t, ps in pieces.items():
        c_first, c_last = run_of(iters, grid, t * kblocks), run_of(iters, grid, (t + 1) * kblocks - 1)
        assert [p[0] for p in ps] == list(range(c_first, c_last + 1))
        for c, slot, _ in ps:
            assert slot == (0 if run_begin(iters, grid, c) // kblocks == t else 1)
            assert (c, slot) not in slots
            slots.add((c, slot))
        c_close = c_last if run_begin(iters, grid, c_last + 1) <= (t + 1) * kblocks else c_last - 1
        assert c_close >= c_first, "a split tile has at least one closer"
        assert [p[0] for p in ps if p[2]] == list(range(c_first, c_close + 1))
