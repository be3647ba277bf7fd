"""Pin the CPU codec oracle (oracle/codec.py, oracle/decode.c) to the reference.

Records and LUTs in tests/golden/codec.npz were produced by the reference's own
``codec.encode`` (tests/golden/make_golden.py).  No GPU needed.
"""

import os

import numpy as np
import pytest

from digest import digest
from oracle import _lib
from oracle import codec as oc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def g():
    return np.load(os.path.join(GOLDEN, "codec.npz"))


def test_code_lengths_match_reference(g):
    for hist, want in zip(g["hists"], g["lengths"]):
        got = oc.code_lengths(hist.tolist())
        assert got == want.tolist()
        assert max(got) <= oc.LIMIT
        assert sum(2.0 ** -n for n in got) == 1.0


@pytest.mark.parametrize("chunk", [64, 512])
@pytest.mark.parametrize("i", range(4), ids=["realistic", "uniform", "geometric", "constant"])
def test_encode_matches_reference_bytes(g, chunk, i):
    raw = g[f"c{chunk}_{i}_raw"]
    rec, lut, used = oc.encode(raw, g[f"c{chunk}_{i}_rec"].size, chunk)
    assert np.array_equal(rec, g[f"c{chunk}_{i}_rec"])
    assert np.array_equal(lut, g[f"c{chunk}_{i}_lut"])
    assert used == int(g[f"c{chunk}_{i}_used"])


@pytest.mark.parametrize("chunk", [64, 512])
@pytest.mark.parametrize("i", range(4), ids=["realistic", "uniform", "geometric", "constant"])
def test_decoders_invert_reference_records(g, chunk, i):
    raw = g[f"c{chunk}_{i}_raw"]
    rec, lut = g[f"c{chunk}_{i}_rec"], g[f"c{chunk}_{i}_lut"]
    assert np.array_equal(_lib.decode(rec, lut, raw.size, chunk), raw)
    if chunk == 64 and i < 2:  # the pure-Python decoder is slow; two cases suffice
        assert np.array_equal(oc.decode_py(rec, lut, raw.size, chunk), raw)


def test_encode_rejects_rows_over_pitch(g):
    raw = g["c64_0_raw"]
    with pytest.raises(ValueError) as e:
        oc.encode(raw, raw.size // 4, 64)
    assert "VLLM_EXPERT_PAGER_PITCH must be at least" in str(e.value)
    with pytest.raises(ValueError, match="not a multiple"):
        oc.encode(np.zeros(raw.size + 8, np.uint8), 8 * raw.size, 64)


def test_over_pitch_message_matches_reference(g):
    # the reference message for the test_codec.py rows(3) case at CHUNK=64
    from rowgen import rows

    raw = rows(3, 4096).numpy()
    with pytest.raises(ValueError) as e:
        oc.encode(raw, 1024, 64)
    assert str(e.value) == str(g["over_pitch_msg"])


def test_config1_records_match_reference(g):
    """Config 1: 8 experts x (w13, w2), encoded at pitch 0.89 and decoded back."""
    import torch

    from vllm_expert_pager import synthetic

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    experts = synthetic.fp8_experts(8, seed=0)
    for e, ex in enumerate(experts):
        for k, name in enumerate(synthetic.SHAPES):
            q, scale = ex[name]
            raw = synthetic.row_bytes(q).numpy()
            want = list(g["cfg1_digests"][e][k])
            assert digest(raw) == want[0] and digest(scale.view(torch.int32)) == want[1]
            pitch = oc.pitch_of(raw.size, 0.89, 4096)
            assert pitch == int(g["cfg1_pitch"][k])
            rec, lut, used = oc.encode(raw, pitch)
            assert digest(rec) == want[2], f"expert {e} {name}"
            assert np.array_equal(lut, g["cfg1_luts"][e][k])
            assert used == int(g["cfg1_used"][e][k])
            if e < 2:
                assert np.array_equal(_lib.decode(rec, lut, raw.size), raw)
