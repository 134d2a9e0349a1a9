"""Flat parameter / gradient / optimizer-state storage.

All parameters of a model live in ONE fp32 master buffer (with a bf16 mirror
for the tensor-core kernels), one fp32 gradient buffer and the optimizer
moments, so that the fused optimizer updates the whole model in a single
launch and gradient buckets for the data-parallel all-reduce are plain
contiguous slices. Every tensor starts on a 64-element boundary (256-byte
aligned in fp32), which keeps vector loads and TMA descriptors aligned and
lets a one-byte-per-64-elements mask carry per-tensor weight-decay flags.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

ALIGN = 64


def _round_up(x: int, a: int = ALIGN) -> int:
    return (x + a - 1) // a * a


@dataclass
class Slot:
    name: str
    shape: tuple
    offset: int
    numel: int
    decay: bool


class FlatParams:
    """Registry + storage. Call `add` for every tensor, then `allocate`."""

    def __init__(self):
        self.slots: dict[str, Slot] = {}
        self.order: list[str] = []
        self.total = 0
        self.master = self.p16 = self.grad = None
        self.decay_mask = None

    def add(self, name: str, shape, decay: bool) -> Slot:
        shape = tuple(int(s) for s in shape)
        n = 1
        for s in shape:
            n *= s
        slot = Slot(name, shape, self.total, n, decay)
        self.slots[name] = slot
        self.order.append(name)
        self.total += _round_up(n)
        return slot

    def pad_to(self, multiple: int) -> int:
        """Advance the end offset to a multiple of `multiple` elements (e.g.
        so that gradient buckets split evenly into per-rank shards)."""
        self.total = _round_up(self.total, int(multiple))
        return self.total

    def mark(self) -> int:
        """Current end offset (use to delimit gradient buckets)."""
        return self.total

    def allocate(self, device, with_bf16: bool = True):
        n = self.total
        self.master = torch.zeros(n, dtype=torch.float32, device=device)
        self.grad = torch.zeros(n, dtype=torch.float32, device=device)
        self.p16 = torch.zeros(n, dtype=torch.bfloat16, device=device) if with_bf16 else None
        mask = torch.zeros((n + ALIGN - 1) // ALIGN, dtype=torch.uint8)
        for s in self.slots.values():
            if s.decay:
                mask[s.offset // ALIGN : (s.offset + _round_up(s.numel)) // ALIGN] = 1
        self.decay_mask = mask.to(device)
        return self

    def view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        s = self.slots[name]
        return buf[s.offset : s.offset + s.numel].view(s.shape)

    def w(self, name):  # bf16 weights for the kernels
        return self.view(self.p16, name)

    def m(self, name):  # fp32 master
        return self.view(self.master, name)

    def g(self, name):  # fp32 gradient
        return self.view(self.grad, name)

    def sync_bf16(self):
        if self.p16 is not None:
            self.p16.copy_(self.master)

    def state_dict(self) -> dict[str, torch.Tensor]:
        return {k: self.m(k).detach().clone() for k in self.order}

    def load_state_dict(self, sd: dict[str, torch.Tensor]):
        for k in self.order:
            if k in sd:
                self.m(k).copy_(sd[k].reshape(self.slots[k].shape))
        self.sync_bf16()
