"""Recurrent layers: RNN, LSTM, GRU, Bidirectional
(scirs2-neural/src/layers/recurrent/*.rs). Batch-first [B, S, F] inputs;
PyTorch's fused recurrent kernels do the time loop (cuDNN on GPU)."""
from __future__ import annotations

import torch
import torch.nn as nn

from .base import Layer


class _Rec(Layer):
    cell = None

    def __init__(self, input_size: int, hidden_size: int, num_layers: int = 1, return_sequences: bool = True,
                 dtype=torch.float32, device=None):
        super().__init__()
        self.rnn = type(self).cell(input_size, hidden_size, num_layers, batch_first=True, dtype=dtype, device=device)
        self.return_sequences = return_sequences
        self.hidden_size = hidden_size

    def forward(self, x, state=None):
        y, st = self.rnn(x, state)
        self.last_state = st
        return y if self.return_sequences else y[:, -1]


class RNN(_Rec):
    cell = nn.RNN


class LSTM(_Rec):
    cell = nn.LSTM


class GRU(_Rec):
    cell = nn.GRU


class Bidirectional(Layer):
    """Runs a recurrent layer forward and on the time-reversed input and
    concatenates (or sums) the two output sequences."""

    def __init__(self, forward_layer: _Rec, backward_layer: _Rec | None = None, merge: str = "concat"):
        super().__init__()
        import copy

        self.fwd = forward_layer
        self.bwd = backward_layer if backward_layer is not None else copy.deepcopy(forward_layer)
        self.merge = merge

    def forward(self, x):
        a = self.fwd(x)
        b = self.bwd(torch.flip(x, [1]))
        if b.dim() == 3:
            b = torch.flip(b, [1])
        return torch.cat([a, b], -1) if self.merge == "concat" else a + b
