import pytest
import torch

from scirs_b200.export.weights import WeightFormat, WeightStore, pytorch_to_scirs2_names, scirs2_to_pytorch_names


def _store():
    s = WeightStore()
    s.insert("fc.weight", torch.arange(32, dtype=torch.float64).view(4, 8) / 7)
    s.insert("fc.bias", torch.zeros(4))
    s.set_metadata("framework", "scirs_b200")
    return s


@pytest.mark.parametrize("fmt", list(WeightFormat))
def test_round_trip(tmp_path, fmt):
    s = _store()
    p = str(tmp_path / f"w.{fmt.value}")
    s.save(p, fmt)
    t = WeightStore.load(p, fmt)
    assert t.names() == s.names() and t.get_metadata("framework") == "scirs_b200"
    assert all(torch.equal(t.get(k), s.get(k)) for k in s.names())
    if fmt is WeightFormat.NPZ_LIKE:
        assert (tmp_path / f"w.{fmt.value}.idx.json").exists()


def test_names_validation_upcast():
    s = _store()
    r = s.rename_with(pytorch_to_scirs2_names)
    assert r.get("fc.kernel") is not None and r.get("fc.weight") is None
    assert pytorch_to_scirs2_names("bn.num_batches_tracked") == ""
    assert pytorch_to_scirs2_names("bn.running_mean") == "bn.mean"
    assert scirs2_to_pytorch_names("bn.var") == "bn.running_var" and scirs2_to_pytorch_names("fc.kernel") == "fc.weight"
    s.validate_shapes({"fc.weight": [4, 8], "fc.bias": [4]})
    with pytest.raises(ValueError):
        s.validate_shapes({"fc.weight": [8, 4]})
    with pytest.raises(KeyError):
        s.validate_shapes({"nope": [1]})
    u = s.upcast_f32()
    assert torch.equal(u.get("fc.weight"), s.get("fc.weight").float().double())
    m = torch.nn.Sequential(torch.nn.Linear(3, 2), torch.nn.BatchNorm1d(2))
    ws = WeightStore.from_module(m, pytorch_to_scirs2_names)
    assert "1.mean" in ws.names() and "0.kernel" in ws.names() and len(ws) == 6
