"""The packed refinement records (`index_build.pack_records`) are byte-identical to the reference's
`tiered_fused.pack` on the golden tiered codes (throughput-mode uniform code and default-engine Lloyd-Max code)."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, pkg


@pytest.mark.parametrize("tag,name", [("i8_", "i8_reference.npz"), ("tr_", "trellis_reference.npz")])
def test_pack_records_match_reference(tag, name):
    ref = np.load(os.path.join(GOLDEN, "pack_reference.npz"))
    f = np.load(os.path.join(GOLDEN, name))
    TS = [tuple(int(v) for v in r) for r in f["TS"]]
    planes = [torch.from_numpy(f[f"planes{t}"]) for t in range(len(TS))]
    rec, RB, soff, toff = pkg("index_build").pack_records(TS, planes, torch.from_numpy(f["scale"]),
                                                          torch.from_numpy(f["sig"]))
    assert RB == int(ref[tag + "RB"]) and soff == int(ref[tag + "soff"])
    assert list(toff) == list(ref[tag + "toff"])
    np.testing.assert_array_equal(rec.numpy(), ref[tag + "rec"])
