import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle

    oracle.build()
    return oracle


# Every greedy-sequence comparison of the session: (test, steps, smallest
# oracle top-2 margin met, step where the near-tie allowance fired or None).
_GREEDY_REPORT = []


class GreedyCheck:
    """Greedy ids of the GPU against the CPU oracle (generate's argmax loop,
    src/model.rs:614-663 with argmax, src/tensor.rs:1063-1073).

    The bar is identical ids.  One allowance: at a step whose top-2 logits
    differ by less than NEAR_TIE in the oracle, the pick is decided by
    summation order (the GPU's parallel sums differ from the reference's
    sequential ones in the last bits); there the GPU may take the oracle's
    runner-up, and the sequences are compared up to that step only.  Every
    comparison is reported at the end of the session with the smallest
    margin it met and whether (and where) the allowance fired."""

    NEAR_TIE = 1e-3

    @staticmethod
    def oracle(om, prompt, n):
        """The oracle's greedy ids with, per step, the top-2 margin and the
        runner-up id (the prompt is prefilled into a fresh cache)."""
        om.reset()
        logits = om.forward_seq(prompt)
        first = logits.copy()
        ids, margins, second = [], [], []
        for _ in range(n):
            top = np.argsort(-logits, kind="stable")[:2]
            ids.append(int(top[0]))
            margins.append(float(logits[top[0]] - logits[top[1]]))
            second.append(int(top[1]))
            logits = om.forward_token(int(top[0]))
        return ids, margins, second, first

    def agree(self, name, gpu, ref, margins, second, near_tie=None):
        """near_tie: the margin below which a flip is allowed (NEAR_TIE
        unless a test states a wider one, with its reason)."""
        tie = self.NEAR_TIE if near_tie is None else near_tie
        gpu = [int(t) for t in gpu]
        assert len(gpu) == len(ref), (len(gpu), len(ref))
        i = next((j for j, (a, b) in enumerate(zip(gpu, ref)) if a != b), None)
        upto = len(ref) if i is None else i + 1
        _GREEDY_REPORT.append((name, len(ref), min(margins[:upto]), i))
        if i is None:
            return
        assert margins[i] < tie and gpu[i] == second[i], (
            f"{name}: greedy diverged at step {i} (oracle margin {margins[i]:.2e}): gpu {gpu[i]} "
            f"vs oracle {ref[i]} (runner-up {second[i]})")


@pytest.fixture(scope="session")
def greedy():
    return GreedyCheck()


def pytest_terminal_summary(terminalreporter):
    if not _GREEDY_REPORT:
        return
    terminalreporter.section("greedy parity against the oracle")
    for name, n, m, i in _GREEDY_REPORT:
        how = "identical" if i is None else f"near-tie allowance used at step {i}"
        terminalreporter.write_line(f"{name}: {n} steps, smallest oracle top-2 margin {m:.3e}, {how}")
