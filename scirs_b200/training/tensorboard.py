"""TensorBoard event files: writer, reader and a training callback.

Files follow TensorBoard's on-disk format so `tensorboard --logdir` reads
them: a sequence of records, each

    uint64 length | uint32 masked_crc32c(length bytes) | data | uint32 masked_crc32c(data)

(little endian; masked(c) = ((c >> 15) | (c << 17)) + 0xa282ead8 mod 2^32),
where every `data` is a serialized `Event` protobuf: wall_time (1, double),
step (2, int64), file_version (3, string, first record "brain.Event:2") or
summary (5, Summary). Summary holds repeated Value (1) = {tag (1),
simple_value (2, float) | histo (5, HistogramProto{min 1, max 2, num 3,
sum 4, sum_squares 5, bucket_limit 6, bucket 7})}. The protobuf bytes and
the CRC-32C (Castagnoli polynomial 0x82F63B78, reflected, table driven) are
produced here; no TensorFlow or tensorboard package is needed.

Reference parity: scirs2-neural/src/callbacks/tensorboard.rs:14-120
(TensorBoardLogger{log_dir, log_histograms, update_freq}; a printing
placeholder there).
"""
from __future__ import annotations

import os
import socket
import struct
import time

import torch

from .history import Callback

# ------------------------------------------------------------------ CRC-32C
_POLY = 0x82F63B78


def _make_table():
    t = []
    for i in range(256):
        c = i
        for _ in range(8):
            c = (c >> 1) ^ _POLY if c & 1 else c >> 1
        t.append(c)
    return t


_TABLE = _make_table()


def crc32c(data: bytes) -> int:
    c = 0xFFFFFFFF
    for b in data:
        c = _TABLE[(c ^ b) & 0xFF] ^ (c >> 8)
    return c ^ 0xFFFFFFFF


def masked_crc(data: bytes) -> int:
    c = crc32c(data)
    return (((c >> 15) | (c << 17)) + 0xA282EAD8) & 0xFFFFFFFF


# ------------------------------------------------------------ protobuf bits
def _varint(n: int) -> bytes:
    n &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = n & 0x7F
        n >>= 7
        out.append(b | (0x80 if n else 0))
        if not n:
            return bytes(out)


def _key(f: int, wire: int) -> bytes:
    return _varint((f << 3) | wire)


def _ld(f: int, payload: bytes) -> bytes:
    return _key(f, 2) + _varint(len(payload)) + payload


def _double(f: int, v: float) -> bytes:
    return _key(f, 1) + struct.pack("<d", float(v))


def _float(f: int, v: float) -> bytes:
    return _key(f, 5) + struct.pack("<f", float(v))


def _packed_doubles(f: int, vals) -> bytes:
    return _ld(f, b"".join(struct.pack("<d", float(v)) for v in vals))


def _histogram_proto(values: torch.Tensor, bins: int) -> bytes:
    v = values.detach().double().reshape(-1).cpu()
    v = v[torch.isfinite(v)]
    if v.numel() == 0:
        v = torch.zeros(1, dtype=torch.float64)
    lo, hi = float(v.min()), float(v.max())
    if hi <= lo:
        hi = lo + 1e-12
    counts = torch.histc(v, bins=bins, min=lo, max=hi)
    edges = torch.linspace(lo, hi, bins + 1)[1:].tolist()
    edges[-1] = max(edges[-1], hi)
    b = _double(1, lo) + _double(2, hi) + _double(3, float(v.numel())) + _double(4, float(v.sum()))
    b += _double(5, float((v * v).sum()))
    return b + _packed_doubles(6, edges) + _packed_doubles(7, counts.tolist())


def _event(wall: float, step: int, file_version: str | None = None, summary: bytes | None = None) -> bytes:
    b = _double(1, wall) + _key(2, 0) + _varint(int(step))
    if file_version is not None:
        b += _ld(3, file_version.encode())
    if summary is not None:
        b += _ld(5, summary)
    return b


def _record(data: bytes) -> bytes:
    n = struct.pack("<Q", len(data))
    return n + struct.pack("<I", masked_crc(n)) + data + struct.pack("<I", masked_crc(data))


# ------------------------------------------------------------------- writer
class EventFileWriter:
    """Appends TensorBoard events to `log_dir/events.out.tfevents.<time>.<host>`."""

    def __init__(self, log_dir: str, filename_suffix: str = ""):
        os.makedirs(log_dir, exist_ok=True)
        self.path = os.path.join(
            log_dir, f"events.out.tfevents.{int(time.time())}.{socket.gethostname()}{filename_suffix}")
        self.f = open(self.path, "ab")
        self.f.write(_record(_event(time.time(), 0, file_version="brain.Event:2")))
        self.f.flush()

    def _write(self, step: int, value: bytes):
        self.f.write(_record(_event(time.time(), step, summary=_ld(1, value))))

    def add_scalar(self, tag: str, value: float, step: int):
        self._write(step, _ld(1, tag.encode()) + _float(2, float(value)))

    def add_scalars(self, values: dict, step: int):
        for k, v in values.items():
            self.add_scalar(k, v, step)

    def add_histogram(self, tag: str, values: torch.Tensor, step: int, bins: int = 64):
        self._write(step, _ld(1, tag.encode()) + _ld(5, _histogram_proto(values, bins)))

    def flush(self):
        self.f.flush()

    def close(self):
        if not self.f.closed:
            self.f.flush()
            self.f.close()


# ------------------------------------------------------------------- reader
def _fields(b: bytes):
    i = 0
    while i < len(b):
        k, i = _rd_varint(b, i)
        f, w = k >> 3, k & 7
        if w == 0:
            v, i = _rd_varint(b, i)
        elif w == 1:
            v, i = b[i:i + 8], i + 8
        elif w == 5:
            v, i = b[i:i + 4], i + 4
        elif w == 2:
            n, i = _rd_varint(b, i)
            v, i = b[i:i + n], i + n
        else:
            raise ValueError(f"unsupported wire type {w}")
        yield f, w, v


def _rd_varint(b: bytes, i: int):
    r = s = 0
    while True:
        c = b[i]
        i += 1
        r |= (c & 0x7F) << s
        s += 7
        if not c & 0x80:
            return r, i


def read_events(path: str) -> list[dict]:
    """Parse an event file (checking both CRCs of every record). Returns one
    dict per event: {"wall_time", "step", "file_version" | "scalars" |
    "histograms"}."""
    out = []
    data = open(path, "rb").read()
    i = 0
    while i < len(data):
        head = data[i:i + 8]
        (n,) = struct.unpack("<Q", head)
        (hc,) = struct.unpack("<I", data[i + 8:i + 12])
        if hc != masked_crc(head):
            raise ValueError(f"corrupt length CRC at byte {i}")
        body = data[i + 12:i + 12 + n]
        (bc,) = struct.unpack("<I", data[i + 12 + n:i + 16 + n])
        if bc != masked_crc(body):
            raise ValueError(f"corrupt data CRC at byte {i}")
        i += 16 + n
        ev = {"scalars": {}, "histograms": {}}
        for f, _, v in _fields(body):
            if f == 1:
                ev["wall_time"] = struct.unpack("<d", v)[0]
            elif f == 2:
                ev["step"] = v
            elif f == 3:
                ev["file_version"] = v.decode()
            elif f == 5:
                for _, _, val in _fields(v):
                    tag, sv, hist = None, None, None
                    for vf, _, vv in _fields(val):
                        if vf == 1:
                            tag = vv.decode()
                        elif vf == 2:
                            sv = struct.unpack("<f", vv)[0]
                        elif vf == 5:
                            hist = _read_hist(vv)
                    if sv is not None:
                        ev["scalars"][tag] = sv
                    if hist is not None:
                        ev["histograms"][tag] = hist
        out.append(ev)
    return out


def _read_hist(b: bytes) -> dict:
    h = {"bucket_limit": [], "bucket": []}
    names = {1: "min", 2: "max", 3: "num", 4: "sum", 5: "sum_squares"}
    for f, _, v in _fields(b):
        if f in names:
            h[names[f]] = struct.unpack("<d", v)[0]
        elif f in (6, 7):
            vals = list(struct.unpack("<%dd" % (len(v) // 8), v))
            h["bucket_limit" if f == 6 else "bucket"] += vals
    return h


# ----------------------------------------------------------------- callback
class TensorBoardLogger(Callback):
    """Logs batch losses every `update_freq` batches, every epoch metric, and
    (with `log_histograms`) a histogram of every parameter and its gradient
    at the end of each epoch."""

    def __init__(self, log_dir: str, log_histograms: bool = False, update_freq: int = 1):
        self.writer = EventFileWriter(log_dir)
        self.log_histograms = log_histograms
        self.update_freq = max(1, int(update_freq))
        self.global_step = 0

    def on_batch_end(self, step, model, logs=None):
        self.global_step += 1
        if logs and self.global_step % self.update_freq == 0:
            for k, v in logs.items():
                if isinstance(v, (int, float)) or (torch.is_tensor(v) and v.numel() == 1):
                    self.writer.add_scalar(f"batch/{k}", float(v), self.global_step)

    def on_epoch_end(self, epoch, model, logs=None):
        for k, v in (logs or {}).items():
            if v is not None:
                self.writer.add_scalar(f"epoch/{k}", float(v), epoch)
        if self.log_histograms and hasattr(model, "named_parameters"):
            for name, p in model.named_parameters():
                self.writer.add_histogram(f"params/{name}", p, epoch)
                if p.grad is not None:
                    self.writer.add_histogram(f"grads/{name}", p.grad, epoch)
        self.writer.flush()

    def on_train_end(self, model, logs=None):
        self.writer.close()
