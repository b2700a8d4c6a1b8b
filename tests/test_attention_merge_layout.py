"""Host-side restatement of the split attention's cluster merge by pushes
(attention.cu, attention_kernel), checked on the CPU for every head shape the
kernel is instantiated for and every cluster size.

After the warps of a CTA merge, thread t holds the CTA's outputs
[hg D + hd, hg D + hd + E) with E = max(G D / 128, 1), hg = t / (D / E),
hd = (t mod (D / E)) E, when hg < G. CTA q of a cluster of csize owns outputs
[q per, min(G D, (q + 1) per)), per = ceil(G D / csize). Every CTA c sends each
of its outputs i to owner q = i / per at recv_o[c per + i - q per], and thread
t < csize G sends the (m, l) of head t mod G to owner t / G at
recv_ml[(c G + h) 2]. The owner's mbarrier expects csize (hi - lo + 2 G) x 4
bytes. Checked: every output has exactly one sending thread; every owner
receives each of its slots from each CTA exactly once, and the bytes it
receives equal the bytes it expects (a mismatch would leave it waiting until
its bounded wait ran out); all indices stay inside the receive buffers.
"""

import pytest

THREADS = 128
MAX_CLUSTER = 16


def sends(G, D, csize, crank):
    """(owner, 'o' or 'ml', buffer index, bytes) of every store CTA crank issues."""
    E = max(G * D // THREADS, 1)
    per = (G * D + csize - 1) // csize
    out = []
    for t in range(THREADS):
        hg, hd = t // (D // E), (t % (D // E)) * E
        if hg < G:
            for e in range(E):
                i = hg * D + hd + e
                q = i // per
                out.append((q, "o", crank * per + i - q * per, 4))
        if t < csize * G:
            q, h = t // G, t % G
            out.append((q, "ml", (crank * G + h) * 2, 8))
    return out


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("csize", [1, 2, 4, 8, 16])
def test_push_merge_slots_and_bytes(G, D, csize):
    assert MAX_CLUSTER * G <= THREADS  # the kernel's static_assert: one (m, l) send per thread
    per = (G * D + csize - 1) // csize
    # each output is sent by exactly one thread of a CTA
    E = max(G * D // THREADS, 1)
    owners = {}
    for t in range(THREADS):
        hg, hd = t // (D // E), (t % (D // E)) * E
        if hg < G:
            for e in range(E):
                owners.setdefault(hg * D + hd + e, []).append(t)
    assert sorted(owners) == list(range(G * D))
    assert all(len(v) == 1 for v in owners.values())
    received = {q: {"o": [], "ml": [], "bytes": 0} for q in range(csize)}
    for c in range(csize):
        for q, kind, idx, nbytes in sends(G, D, csize, c):
            assert 0 <= q < csize
            received[q][kind].append(idx)
            received[q]["bytes"] += nbytes
    for q in range(csize):
        lo, hi = q * per, min(G * D, (q + 1) * per)
        width = max(hi - lo, 0)
        expect_o = sorted(c * per + k for c in range(csize) for k in range(width))
        assert sorted(received[q]["o"]) == expect_o
        assert sorted(received[q]["ml"]) == sorted((c * G + h) * 2 for c in range(csize) for h in range(G))
        assert received[q]["bytes"] == csize * (width + 2 * G) * 4  # the owner's expect_tx
        assert max(received[q]["o"], default=0) < G * D + MAX_CLUSTER  # recv_o size
        assert max(received[q]["ml"]) + 1 < MAX_CLUSTER * G * 2  # recv_ml size
