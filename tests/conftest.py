import importlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pkg(name=None):
    """The product package (its directory name has a hyphen, so it is loaded through importlib)."""
    return importlib.import_module("fanarvse-paper_b200" + ("." + name if name else ""))


@pytest.fixture(scope="session")
def golden_i8():
    return dict(np.load(os.path.join(GOLDEN, "i8_reference.npz")))


def golden_index(f, case):
    """Index dict (oracle layout) of one golden case."""
    TS = [tuple(int(v) for v in r) for r in f["TS"]]
    code = dict(TS=TS, planes=[f[f"planes{t}"] for t in range(len(TS))], scale=f["scale"], sig=f["sig"],
                VP16=f["VP16"], deltas={TS[t][2]: float(f["deltas"][t]) for t in range(len(TS))})
    return dict(off=f[case + "s1_off"], order=f["order"], means16=f[case + "s1_means16"],
                inv_mnorm=f[case + "s1_inv_mnorm"], c=f["c"], Z=f["Z"], zs=f["zs"], Vr=f["Vr"], code=code,
                H16=f["H16"])


def assert_end_to_end(g, o, z, k):
    """End-to-end parity of a search against the oracle (or the reference's goldens) on the same inputs.

    g / o: dicts with ok, t0, cnt, ids, reads, I, est, sd (numpy).  On every row both sides accept (ok): where the
    ambiguous sets agree the final ids are identical; where they differ, every candidate that differs lies within 1e-5
    (relative) of a classification boundary on one side's fp32 stage-2 sums -- a last-bit rounding of those sums, not a
    different candidate set.  Returns the report (counts per output)."""
    from oracle import fvs_oracle as O
    rep = O.parity_report(g, o, z, k)
    assert rep["I_equal_where_amb_equal"] == rep["amb_sets_equal"], rep
    assert rep["amb_differs_explained"] == rep["amb_differs"], rep
    return rep
