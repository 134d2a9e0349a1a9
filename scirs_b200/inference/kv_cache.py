"""Paged key/value cache for decoding on the GPU.

A :class:`KvPagePool` owns two device tensors [num_pages, block_size, Hkv, HD]
(bf16) and a host free list; a page id names one page in both. The
:class:`BlockManager` maps sequence ids to page chains, grows them as tokens
are appended, and keeps the device block table (int32 [max_sequences,
max_pages_per_seq]) that the decode kernel reads. Appending the K/V of any
number of tokens of any sequences is one kernel launch.

Names and semantics follow the reference's inference module
(scirs2-neural/src/inference/kv_page.rs:27-340 KvPageConfig / KvPage /
KvPagePool, block_manager.rs:30-280 BlockManagerConfig / BlockManager /
SharedPrefixCache); there the pages are ndarray buffers on the host.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch

from .. import _ext


class InferenceError(RuntimeError):
    pass


@dataclass
class KvPageConfig:
    block_size: int = 16
    num_heads: int = 8
    head_dim: int = 64
    dtype_bytes: int = 2

    @property
    def page_bytes(self) -> int:
        return 2 * self.block_size * self.num_heads * self.head_dim * self.dtype_bytes


class KvPagePool:
    def __init__(self, num_pages: int, config: KvPageConfig, device="cuda"):
        c = config
        self.config = c
        self.device = torch.device(device)
        shape = (num_pages, c.block_size, c.num_heads, c.head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self._free = list(range(num_pages - 1, -1, -1))
        self._used: set[int] = set()
        self._tick = 0
        self._last_use: dict[int, int] = {}

    def alloc_page(self) -> int:
        if not self._free:
            raise InferenceError("KV page pool exhausted")
        pid = self._free.pop()
        self._used.add(pid)
        self._touch(pid)
        return pid

    def free_page(self, pid: int) -> None:
        if pid not in self._used:
            raise InferenceError(f"page {pid} is not allocated")
        self._used.remove(pid)
        self._last_use.pop(pid, None)
        self._free.append(pid)

    def _touch(self, pid: int):
        self._tick += 1
        self._last_use[pid] = self._tick

    def free_count(self) -> int:
        return len(self._free)

    def total_count(self) -> int:
        return self.k.shape[0]

    def memory_bytes(self) -> int:
        return self.total_count() * self.config.page_bytes

    def lru_candidates(self):
        """Allocated pages, least recently written first."""
        return [p for p, _ in sorted(self._last_use.items(), key=lambda kv: kv[1])]

    def write_kv(self, pid: int, slot: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Write one token's K/V ([Hkv, HD]) into a page slot (host-driven
        path; the batched path is BlockManager.append)."""
        if pid not in self._used or not 0 <= slot < self.config.block_size:
            raise InferenceError("slot out of range")
        self.k[pid, slot].copy_(k)
        self.v[pid, slot].copy_(v)
        self._touch(pid)

    def read_kv(self, pid: int, slot: int):
        return self.k[pid, slot], self.v[pid, slot]


@dataclass
class BlockManagerConfig:
    max_sequences: int = 64
    max_pages_per_seq: int = 128


class BlockManager:
    def __init__(self, pool: KvPagePool, config: BlockManagerConfig | None = None):
        self.pool = pool
        self.config = config or BlockManagerConfig()
        c = self.config
        self.block_tables = torch.zeros(c.max_sequences, c.max_pages_per_seq, dtype=torch.int32,
                                        device=pool.device)
        self._bt_host = torch.zeros(c.max_sequences, c.max_pages_per_seq, dtype=torch.int32)
        self.seq_lens = torch.zeros(c.max_sequences, dtype=torch.int32, device=pool.device)
        self._lens: dict[int, int] = {}
        self._pages: dict[int, list[int]] = {}
        self._row: dict[int, int] = {}
        self._free_rows = list(range(c.max_sequences - 1, -1, -1))
        self._dirty = False

    # ---------------------------------------------------------------- chains
    def allocate_sequence(self, seq_id: int) -> None:
        if seq_id in self._pages:
            raise InferenceError(f"sequence {seq_id} already exists")
        if not self._free_rows:
            raise InferenceError("too many active sequences")
        self._row[seq_id] = self._free_rows.pop()
        self._pages[seq_id] = []
        self._lens[seq_id] = 0
        try:
            self.extend_sequence(seq_id)
        except InferenceError:  # no page for it: leave no half-created sequence behind
            self._free_rows.append(self._row.pop(seq_id))
            del self._pages[seq_id], self._lens[seq_id]
            raise

    def extend_sequence(self, seq_id: int) -> int:
        pages = self._pages[seq_id]
        if len(pages) >= self.config.max_pages_per_seq:
            raise InferenceError("sequence exceeds max_pages_per_seq")
        pid = self.pool.alloc_page()
        self._bt_host[self._row[seq_id], len(pages)] = pid
        pages.append(pid)
        self._dirty = True
        return pid

    def free_sequence(self, seq_id: int) -> None:
        for pid in self._pages.pop(seq_id):
            self.pool.free_page(pid)
        row = self._row.pop(seq_id)
        self._lens.pop(seq_id)
        self._bt_host[row].zero_()
        self._free_rows.append(row)
        self._dirty = True

    def sequence_page_chain(self, seq_id: int) -> list[int]:
        return list(self._pages[seq_id])

    def seq_len(self, seq_id: int) -> int:
        return self._lens[seq_id]

    def row_of(self, seq_id: int) -> int:
        return self._row[seq_id]

    def active_sequences(self) -> int:
        return len(self._pages)

    def sync(self):
        """Upload the block table and lengths if they changed."""
        if self._dirty:
            self.block_tables.copy_(self._bt_host, non_blocking=True)
            lens = torch.zeros(self.config.max_sequences, dtype=torch.int32)
            for s, n in self._lens.items():
                lens[self._row[s]] = n
            self.seq_lens.copy_(lens, non_blocking=True)
            self._dirty = False

    # ---------------------------------------------------------------- writes
    def reserve(self, seq_ids: list[int], counts: list[int]):
        """Grow chains for `counts` new tokens per sequence; returns the
        (row, position) of every new token in order."""
        rows, pos = [], []
        bs = self.pool.config.block_size
        # all or nothing: check the whole batch's page needs before changing any sequence
        need, lens = {}, dict(self._lens)
        for s, n in zip(seq_ids, counts):
            lens[s] += n
            need[s] = max(0, (lens[s] + bs - 1) // bs - len(self._pages[s]))
        if any(len(self._pages[s]) + k > self.config.max_pages_per_seq for s, k in need.items()):
            raise InferenceError("sequence exceeds max_pages_per_seq")
        if sum(need.values()) > self.pool.free_count():
            raise InferenceError("KV page pool exhausted")
        for s, n in zip(seq_ids, counts):
            start = self._lens[s]
            while (start + n + bs - 1) // bs > len(self._pages[s]):
                self.extend_sequence(s)
            rows += [self._row[s]] * n
            pos += list(range(start, start + n))
            self._lens[s] = start + n
            self._dirty = True
        return rows, pos

    def append(self, seq_ids: list[int], counts: list[int], k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Write the K/V ([n, Hkv, HD], n = sum(counts), sequences in order)
        of new tokens into their pages (one kernel launch)."""
        rows, pos = self.reserve(seq_ids, counts)
        self.sync()
        dev = self.pool.device
        r = torch.tensor(rows, dtype=torch.int32).to(dev, non_blocking=True)
        p = torch.tensor(pos, dtype=torch.int32).to(dev, non_blocking=True)
        if k_new.is_cuda:
            _ext.kernels().paged_kv_append(k_new.contiguous(), v_new.contiguous(), self.pool.k, self.pool.v,
                                           self.block_tables, r, p)
        else:
            bs = self.pool.config.block_size
            for i, (row, ps) in enumerate(zip(rows, pos)):
                pid = int(self._bt_host[row, ps // bs])
                self.pool.k[pid, ps % bs] = k_new[i]
                self.pool.v[pid, ps % bs] = v_new[i]

    def write_token_kv(self, seq_id: int, k: torch.Tensor, v: torch.Tensor) -> None:
        self.append([seq_id], [1], k.reshape(1, *k.shape), v.reshape(1, *v.shape))


class SharedPrefixCache:
    """Maps a prompt-prefix hash to the page chain that holds its K/V, so
    sequences with a common prompt can reuse the pages."""

    def __init__(self):
        self._map: dict[int, list[int]] = {}

    def lookup(self, prefix_hash: int):
        return self._map.get(prefix_hash)

    def insert(self, prefix_hash: int, pages: list[int]) -> None:
        self._map[prefix_hash] = list(pages)

    def evict(self, prefix_hash: int):
        return self._map.pop(prefix_hash, None)

    def __len__(self):
        return len(self._map)

    def is_empty(self) -> bool:
        return not self._map

    @staticmethod
    def compute_prefix_hash(tokens) -> int:
        b = b"".join(int(t).to_bytes(4, "little") for t in tokens)
        return int.from_bytes(hashlib.blake2b(b, digest_size=8).digest(), "little")
