"""Out-of-core and chunked array processing for data larger than host or
device memory.

  MemoryMappedArray     a file-backed array (numpy memmap) with torch views of slices;
                        create_mmap / open_mmap / create_temp_mmap
  ChunkedArray          an array processed in chunks along its first axis
  chunk_wise_op         fn applied chunk by chunk, results concatenated
  chunk_wise_binary_op  fn(a_chunk, b_chunk) over two equally shaped arrays
  chunk_wise_reduce     per-chunk map then a reduce over the chunk results
  stream_to_device      yields device tensors of consecutive chunks; on CUDA the next
                        chunk's host->device copy is issued from pinned memory on a side
                        stream while the caller works on the current one

Reference parity: scirs2-core/src/memory_efficient/memmap.rs:68-1260
(MemoryMappedArray, open_mmap, create_mmap, create_temp_mmap),
chunked.rs:316-1080 (ChunkedArray, chunk_wise_op, chunk_wise_binary_op,
chunk_wise_reduce).
"""
from __future__ import annotations

import os
import tempfile

import numpy as np
import torch


class MemoryMappedArray:
    def __init__(self, path: str, shape, dtype=np.float32, mode: str = "r+"):
        self.path, self.shape, self.dtype = path, tuple(int(s) for s in shape), np.dtype(dtype)
        self._mm = np.memmap(path, dtype=self.dtype, mode=mode, shape=self.shape)

    def __len__(self):
        return self.shape[0]

    def to_tensor(self, start: int = 0, stop: int | None = None) -> torch.Tensor:
        """A tensor copy of rows [start, stop)."""
        return torch.from_numpy(np.array(self._mm[start:stop]))

    def write(self, start: int, values):
        v = values.detach().cpu().numpy() if isinstance(values, torch.Tensor) else np.asarray(values)
        self._mm[start:start + v.shape[0]] = v.astype(self.dtype, copy=False)

    def flush(self):
        self._mm.flush()


def create_mmap(path: str, data) -> MemoryMappedArray:
    arr = data.detach().cpu().numpy() if isinstance(data, torch.Tensor) else np.asarray(data)
    m = MemoryMappedArray(path, arr.shape, arr.dtype, mode="w+")
    m._mm[...] = arr
    m.flush()
    return m


def open_mmap(path: str, shape, dtype=np.float32, mode: str = "r") -> MemoryMappedArray:
    expected = int(np.prod(shape)) * np.dtype(dtype).itemsize
    if os.path.getsize(path) < expected:
        raise ValueError(f"{path} holds {os.path.getsize(path)} bytes, {expected} needed for {tuple(shape)}")
    return MemoryMappedArray(path, shape, dtype, mode)


def create_temp_mmap(data) -> MemoryMappedArray:
    fd, path = tempfile.mkstemp(suffix=".mmap")
    os.close(fd)
    return create_mmap(path, data)


class ChunkedArray:
    def __init__(self, data, chunk_size: int):
        if chunk_size < 1:
            raise ValueError("chunk_size must be positive")
        self.data, self.chunk_size = data, int(chunk_size)

    def num_chunks(self) -> int:
        return (len(self.data) + self.chunk_size - 1) // self.chunk_size

    def chunks(self):
        for i in range(0, len(self.data), self.chunk_size):
            c = self.data.to_tensor(i, i + self.chunk_size) if isinstance(self.data, MemoryMappedArray) \
                else torch.as_tensor(self.data[i:i + self.chunk_size])
            yield c

    def map(self, fn):
        return torch.cat([fn(c) for c in self.chunks()])


def chunk_wise_op(data, fn, chunk_size: int):
    return ChunkedArray(data, chunk_size).map(fn)


def chunk_wise_binary_op(a, b, fn, chunk_size: int):
    if len(a) != len(b):
        raise ValueError("arrays must have the same length")
    ca, cb = ChunkedArray(a, chunk_size).chunks(), ChunkedArray(b, chunk_size).chunks()
    return torch.cat([fn(x, y) for x, y in zip(ca, cb)])


def chunk_wise_reduce(data, chunk_fn, reduce_fn, chunk_size: int):
    return reduce_fn([chunk_fn(c) for c in ChunkedArray(data, chunk_size).chunks()])


def stream_to_device(data, chunk_size: int, device):
    """Yield consecutive chunks as tensors on `device`. On CUDA each chunk is staged in pinned host
    memory and copied on a side stream one chunk ahead; the consumer's stream waits for it."""
    device = torch.device(device)
    chunks = ChunkedArray(data, chunk_size).chunks()
    if device.type != "cuda":
        for c in chunks:
            yield c.to(device)
        return
    side = torch.cuda.Stream(device=device)
    main = torch.cuda.current_stream(device)

    def issue(c):
        if c is None:
            return None
        host = c.pin_memory()
        with torch.cuda.stream(side):
            d = host.to(device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(side)
        return d, ev, host

    nxt = issue(next(chunks, None))
    while nxt is not None:
        d, ev, _host = nxt
        nxt = issue(next(chunks, None))
        main.wait_event(ev)
        d.record_stream(main)
        yield d
