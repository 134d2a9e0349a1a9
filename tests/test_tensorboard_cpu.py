"""TensorBoard event files: CRC-32C, record framing, scalar and histogram
events read back, and the logger callback."""
import glob
import struct

import torch

from scirs_b200.training.tensorboard import (EventFileWriter, TensorBoardLogger, crc32c, masked_crc,
                                             read_events)


def test_crc32c_known_vectors():
    assert crc32c(b"123456789") == 0xE3069283  # CRC-32C check value
    assert crc32c(b"") == 0
    assert crc32c(bytes(32)) == 0x8A9136AA  # 32 zero bytes (RFC 3720 test vector)


def test_event_file_roundtrip(tmp_path):
    w = EventFileWriter(str(tmp_path))
    w.add_scalar("loss", 1.25, 3)
    vals = torch.randn(1000, generator=torch.Generator().manual_seed(0))
    w.add_histogram("w", vals, 3, bins=20)
    w.close()
    raw = open(w.path, "rb").read()
    (n,) = struct.unpack("<Q", raw[:8])
    assert struct.unpack("<I", raw[8:12])[0] == masked_crc(raw[:8])
    evs = read_events(w.path)
    assert evs[0]["file_version"] == "brain.Event:2"
    assert evs[1]["step"] == 3 and abs(evs[1]["scalars"]["loss"] - 1.25) < 1e-7
    h = evs[2]["histograms"]["w"]
    assert h["num"] == 1000 and abs(sum(h["bucket"]) - 1000) < 1e-9
    assert abs(h["min"] - float(vals.min())) < 1e-6 and abs(h["sum"] - float(vals.double().sum())) < 1e-6
    assert len(h["bucket_limit"]) == 20


def test_logger_callback(tmp_path):
    model = torch.nn.Linear(4, 3)
    model(torch.randn(2, 4)).sum().backward()
    cb = TensorBoardLogger(str(tmp_path), log_histograms=True, update_freq=2)
    for s in range(4):
        cb.on_batch_end(s, model, {"loss": 1.0 / (s + 1)})
    cb.on_epoch_end(0, model, {"loss": 0.5, "val_loss": 0.7})
    cb.on_train_end(model)
    path = glob.glob(str(tmp_path / "events.out.tfevents.*"))[0]
    evs = read_events(path)
    batch = [e for e in evs if "batch/loss" in e["scalars"]]
    assert [e["step"] for e in batch] == [2, 4]
    hist_tags = {t for e in evs for t in e["histograms"]}
    assert {"params/weight", "params/bias", "grads/weight", "grads/bias"} <= hist_tags
    assert any(abs(e["scalars"].get("epoch/val_loss", -1) - 0.7) < 1e-6 for e in evs)
