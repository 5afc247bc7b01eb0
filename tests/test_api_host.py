"""Host-side API behaviour that mirrors the reference (no GPU)."""
import pytest
import torch

import memintelli_flash_b200 as M
from memintelli_flash_b200.pimpy.data_formats import _decode_gran, padded_tile
from memintelli_flash_b200.crossbar_shard import shard_bounds


def test_engine_validation_mirrors_reference():
    with pytest.raises(ValueError, match="ADC"):
        M.DPETensor(radc=1, device="cpu")
    with pytest.raises(ValueError, match="DAC"):
        M.DPETensor(rdac=1, device="cpu")
    with pytest.raises(ValueError, match="conductance levels"):
        M.DPETensor(g_level=1, device="cpu")
    with pytest.raises(ValueError, match="low conductance"):
        M.DPETensor(HGS=1e-8, LGS=1e-5, device="cpu")
    with pytest.raises(ValueError, match="stuck"):
        M.DPETensor(rate_stuck_HGS=0.6, rate_stuck_LGS=0.6, device="cpu")
    with pytest.raises(ValueError, match="read_variation dict"):
        M.DPETensor(g_level=4, read_variation={0: 0.1}, device="cpu")
    e = M.DPETensor(radc=[4096, 2048], device="cpu")
    assert e.radc_is_list and e.radc.tolist() == [2048, 4096]      # stored flipped (memmat_tensor.py:82-85)


def test_sliced_data_tables():
    s = M.SlicedData(torch.tensor([1, 1, 2, 2, 2]))
    assert s.sliced_max_weights.tolist() == [3, 3, 3, 1, 1]
    assert s.sliced_weights.tolist() == [1, 4, 16, 64, -128]
    with pytest.raises(ValueError, match="first bit"):
        M.SlicedData(torch.tensor([2, 2]))


def test_cpu_device_fails_loudly():
    e = M.DPETensor(device="cpu")
    s = M.SlicedData(torch.tensor([1, 1, 2, 2, 2]), paral_size=(1, 32), quant_gran=(1, 128))
    with pytest.raises(RuntimeError, match="CUDA"):
        s.slice_data_imp(e, torch.randn(4, 64))


def test_decode_granularity():
    assert _decode_gran((1, 128), (1, 32), 400, 500) == [1, 128]
    assert _decode_gran((100, 100), (32, 32), 400, 500) == [128, 128]
    assert _decode_gran("per-row", (1, 32), 30, 90) == [1, 96]
    assert _decode_gran("per-matrix", (32, 32), 90, 50) == [96, 64]
    assert _decode_gran("per-col", (32, 32), 90, 50) == [96, 32]


def test_padded_tile():
    assert padded_tile(32, 0) == 32 and padded_tile(64, 0) == 64 and padded_tile(16, 0) == 32
    assert padded_tile(32, 1) == 32 and padded_tile(16, 1) == 16 and padded_tile(64, 1) == 64
    with pytest.raises(NotImplementedError):
        padded_tile(256, 0)


def test_shard_bounds_partition():
    for n, blk in ((151936, 128), (3072, 128), (1000, 64), (100, 128)):
        for world in (1, 2, 4, 8):
            spans = [shard_bounds(n, blk, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            for a, b in spans:
                assert a % blk == 0 or a == n
