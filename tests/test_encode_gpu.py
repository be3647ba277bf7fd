"""GPU encoder (encode_gpu.cu via xp_encode_rows) writes the reference's records byte for byte.

Checked against records and LUTs from the reference's own ``codec.encode``
(tests/golden/codec.npz), against the native host encoder on many exponent
distributions and chunk sizes, in batches, and through a GPU round trip.
"""

import os

import numpy as np
import pytest
import torch

from digest import digest
from oracle import codec as oc
from rowgen import rows
from vllm_expert_pager import codec

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = torch.device("cuda")


@pytest.fixture(scope="module")
def g():
    return np.load(os.path.join(GOLDEN, "codec.npz"))


@pytest.mark.parametrize("chunk", [64, 512])
@pytest.mark.parametrize("i", range(4), ids=["realistic", "uniform", "geometric", "constant"])
def test_gpu_encode_matches_reference(g, chunk, i):
    raw = torch.from_numpy(g[f"c{chunk}_{i}_raw"]).to(DEV)
    rec, lut = codec.encode(raw, g[f"c{chunk}_{i}_rec"].size, chunk)
    assert rec.is_cuda and lut.is_cuda
    assert np.array_equal(rec.cpu().numpy(), g[f"c{chunk}_{i}_rec"])
    assert np.array_equal(lut.cpu().numpy(), g[f"c{chunk}_{i}_lut"])


def test_gpu_encode_config1_batch(g):
    """Config 1: the 8 experts' rows of each name in one batched call."""
    from vllm_expert_pager import synthetic

    experts = synthetic.fp8_experts(8, seed=0)
    for k, name in enumerate(synthetic.SHAPES):
        raws = torch.stack([synthetic.row_bytes(ex[name][0]) for ex in experts]).to(DEV)
        pitch = codec.pitch_of(raws.shape[1], 0.89, 4096)
        recs, luts = codec.encode_rows(raws, pitch)
        for e in range(8):
            assert digest(recs[e].cpu().numpy()) == g["cfg1_digests"][e][k][2], f"expert {e} {name}"
            assert np.array_equal(luts[e].cpu().numpy(), g["cfg1_luts"][e][k])


@pytest.mark.parametrize("seed", range(8))
def test_gpu_encode_random_distributions(seed):
    """Skewed, flat and degenerate histograms, every chunk size, a few rows per batch."""
    rng = np.random.default_rng(seed)
    chunk = [8, 16, 64, 512, 128, 32, 24, 256][seed]
    n = 32 * chunk * int(rng.integers(1, 5))
    batch = []
    for r in range(3):
        p = rng.dirichlet(np.full(16, [0.05, 0.3, 1.0, 5.0, 0.1, 2.0, 0.5, 20.0][seed]))
        batch.append(rows(200 + 10 * seed + r, n, p.tolist()).numpy())
    pitch = oc.pitch_of(n, 1.5, 4096) + 4096
    recs, luts = codec.encode_rows(torch.from_numpy(np.stack(batch)).to(DEV), pitch, chunk)
    for r, raw in enumerate(batch):
        want_rec, want_lut = codec.encode(torch.from_numpy(raw), pitch, chunk)  # host encoder
        assert np.array_equal(recs[r].cpu().numpy(), want_rec.numpy())
        assert np.array_equal(luts[r].cpu().numpy(), want_lut.numpy())
        orec, olut, _ = oc.encode(raw, pitch, chunk)
        assert np.array_equal(recs[r].cpu().numpy(), orec)


def test_gpu_encode_decode_round_trip():
    """Encode and expand on the GPU: the slab rows equal the raw rows."""
    n = 32 * 512 * 4
    raws = torch.stack([rows(300 + r, n) for r in range(6)]).to(DEV)
    pitch = codec.pitch_of(n, 0.95, 4096)
    recs, luts = codec.encode_rows(raws, pitch)
    K = 6
    todo = torch.arange(K, dtype=torch.int64, device=DEV)
    dst = [torch.zeros((K, n), dtype=torch.uint8, device=DEV) for _ in range(2)]
    lut2 = torch.stack([luts, luts], dim=1).contiguous()
    codec.decode_rows(todo, todo, torch.full((K,), -1, dtype=torch.int64, device=DEV),
                      [recs, recs], dst, lut2)
    torch.cuda.synchronize()
    assert torch.equal(dst[0], raws) and torch.equal(dst[1], raws)


def test_gpu_encode_errors(g):
    raw = rows(3, 4096).to(DEV)
    with pytest.raises(ValueError) as e:
        codec.encode(raw, 1024, 64)
    assert str(e.value) == str(g["over_pitch_msg"])
    # In a batch, the first row that does not fit is reported.
    batch = torch.stack([rows(3, 4096), torch.zeros(4096, dtype=torch.uint8)]).to(DEV)
    with pytest.raises(ValueError) as e:
        codec.encode_rows(batch, 1024, 64)
    assert str(e.value) == str(g["over_pitch_msg"])
    with pytest.raises(ValueError, match="not a multiple"):
        codec.encode(torch.zeros(4096 + 8, dtype=torch.uint8, device=DEV), 8 * 4096, 64)
    with pytest.raises(ValueError, match="CUDA"):
        codec.encode_rows(torch.zeros((1, 4096), dtype=torch.uint8), 8 * 4096, 64)
