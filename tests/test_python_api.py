"""Host-side behaviour of the jasper-compatible Python surface (no GPU)."""
import numpy as np
import pytest
import torch

import jasper_b200 as jasper


def test_configs_match_reference_ids():
    assert jasper._resolve_config(jasper.DataType.FLOAT16, 32, jasper.DistanceFunc.L2) == "f16_r32_l2"
    assert jasper._resolve_config(jasper.DataType.FLOAT16, 8, jasper.DistanceFunc.INNER_PRODUCT) == "f16_r8_ip"
    with pytest.raises(ValueError):
        jasper._resolve_config(jasper.DataType.FLOAT16, 24, jasper.DistanceFunc.L2)
    assert len(jasper._CONFIGS) == 8
    assert jasper._resolve_directional_config(
        jasper.DataType.FLOAT16, 64, jasper.DistanceFunc.L2, 16, 960) == "f16_r64_l2_k16_d32678"
    assert jasper._resolve_directional_config(
        jasper.DataType.FLOAT16, 32, jasper.DistanceFunc.INNER_PRODUCT, 4, 128) == "f16_r32_ip_k4_d128"
    assert len(jasper._DIRECTIONAL_CONFIGS) == 16


def test_parse_storage_size():
    assert jasper.parse_storage_size("10GB") == 10 * 10**9
    assert jasper.parse_storage_size("1.5 GiB") == int(1.5 * 2**30)
    assert jasper.parse_storage_size("512MiB") == 512 * 2**20
    assert jasper.parse_storage_size("7B") == 7
    for bad in ["10", "GB", "ten GB", "10PB"]:
        with pytest.raises(ValueError):
            jasper.parse_storage_size(bad)


def test_groundtruth_round_trip(tmp_path):
    ids = torch.randint(0, 1000, (5, 20), dtype=torch.int32)
    d = torch.rand(5, 20)
    p = tmp_path / "gt.bin"
    jasper.save_groundtruth(str(p), ids, d)
    i2, d2 = jasper.read_groundtruth(str(p), k=10)
    assert torch.equal(i2, ids[:, :10]) and torch.equal(d2, d[:, :10])
    with pytest.raises(ValueError):
        jasper.read_groundtruth(str(p), k=21)


def test_read_bin_u8_and_f32(tmp_path):
    x = np.arange(24, dtype=np.uint8).reshape(4, 6)
    p = tmp_path / "a.u8bin"
    p.write_bytes(np.array([4, 6], np.uint32).tobytes() + x.tobytes())
    t = jasper.read_bin(str(p), "u8")
    assert t.dtype == torch.float16 and t.shape == (4, 6) and float(t[3, 5]) == 23.0
    y = np.linspace(-1, 1, 12, dtype=np.float32).reshape(3, 4)
    p2 = tmp_path / "a.fbin"
    p2.write_bytes(np.array([3, 4], np.uint32).tobytes() + y.tobytes())
    assert jasper.read_bin(str(p2), "f32", max_vectors=2).shape == (2, 4)


def test_get_recall():
    gt = torch.tensor([[1, 2, 3], [4, 5, 6]])
    res = torch.tensor([[3, 2, 9], [4, 7, 8]])
    assert jasper.get_recall(gt, res, 3, 2, verbose=False) == pytest.approx(3 / 6)


def test_build_validates_inputs_before_gpu():
    with pytest.raises(ValueError):
        jasper.Graph.build(torch.zeros(10, dtype=torch.float16))
    with pytest.raises(ValueError):
        jasper.Graph.build(torch.zeros(10, 4, dtype=torch.float32))
    with pytest.raises(ValueError):
        jasper.Graph.build(torch.zeros(10, 4, dtype=torch.float16), n_neighbors=12)
