"""The native encoder (xp_encode_row, host code) writes the reference's records byte for byte.

Checked against records and LUTs from the reference's own ``codec.encode``
(tests/golden/codec.npz).  No GPU needed.
"""

import os

import numpy as np
import pytest
import torch

from digest import digest
from vllm_expert_pager import codec

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def g():
    return np.load(os.path.join(GOLDEN, "codec.npz"))


@pytest.mark.parametrize("chunk", [64, 512])
@pytest.mark.parametrize("i", range(4), ids=["realistic", "uniform", "geometric", "constant"])
def test_native_encode_matches_reference(g, chunk, i):
    raw = torch.from_numpy(g[f"c{chunk}_{i}_raw"])
    rec, lut = codec.encode(raw, g[f"c{chunk}_{i}_rec"].size, chunk)
    assert np.array_equal(rec.numpy(), g[f"c{chunk}_{i}_rec"])
    assert np.array_equal(lut.numpy(), g[f"c{chunk}_{i}_lut"])


def test_native_encode_config1(g):
    from vllm_expert_pager import synthetic

    experts = synthetic.fp8_experts(8, seed=0)
    for e, ex in enumerate(experts):
        for k, name in enumerate(synthetic.SHAPES):
            raw = synthetic.row_bytes(ex[name][0])
            pitch = codec.pitch_of(raw.numel(), 0.89, 4096)
            rec, lut = codec.encode(raw, pitch)
            assert digest(rec.numpy()) == g["cfg1_digests"][e][k][2], f"expert {e} {name}"
            assert np.array_equal(lut.numpy(), g["cfg1_luts"][e][k])


def test_native_encode_errors(g):
    from rowgen import rows

    raw = rows(3, 4096)
    with pytest.raises(ValueError) as e:
        codec.encode(raw, 1024, 64)
    assert str(e.value) == str(g["over_pitch_msg"])
    with pytest.raises(ValueError, match="not a multiple"):
        codec.encode(torch.zeros(4096 + 8, dtype=torch.uint8), 8 * 4096, 64)
