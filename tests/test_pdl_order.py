"""Source check of the programmatic-dependent-launch order the decode step relies on.

Every kernel releases its dependents (griddepcontrol.launch_dependents) only
after its own dependency wait (griddepcontrol.wait). Then, when a kernel
starts, every kernel two or more launches back has completed, and the decoder
reads inputs written that far back before its own wait: the O and down GEMVs'
residual rows (GemvParams::early_epilogue_inputs), the attention's positions,
block-table rows and older K/V pages. A kernel that released its dependents
before its wait would turn those reads into races, so this test fails on it.
"""

import os
import re

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "aicompiler-test_b200", "csrc")


def kernels(text):
    """(name, body) of every __global__ function, body up to the next one."""
    starts = [m.start() for m in re.finditer(r"__global__", text)]
    for i, s in enumerate(starts):
        end = starts[i + 1] if i + 1 < len(starts) else len(text)
        body = text[s:end]
        names = [n for n in re.findall(r"(\w+)\s*\(", body[:400]) if not n.startswith("__")]
        yield (names[0] if names else "?"), body


def test_every_release_of_dependents_follows_a_dependency_wait():
    checked = 0
    for fn in sorted(os.listdir(CSRC)):
        if not fn.endswith(".cu"):
            continue
        text = open(os.path.join(CSRC, fn)).read()
        text = re.sub(r"//[^\n]*", "", text)  # comments may mention either call
        for name, body in kernels(text):
            for m in re.finditer(r"pdl_launch_dependents\(\)", body):
                assert "pdl_wait()" in body[:m.start()], f"{fn}: {name} releases its dependents before any wait"
                checked += 1
    assert checked >= 6, checked  # GEMV, row prologue, GEMM, both attention schedules, misc
