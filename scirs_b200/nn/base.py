"""The Layer contract of the framework.

Mirrors the reference's `Layer` / `ParamLayer` traits
(scirs2-neural/src/layers/mod.rs:17-119): forward, backward(input,
grad_output), update(learning_rate), params / gradients / set_params,
set_training / is_training, layer_type, parameter_count,
layer_description. Layers are torch.nn.Modules, so autograd provides the
backward pass; `backward()` here is the explicit vector-Jacobian product the
reference exposes, computed through autograd.
"""
from __future__ import annotations

import torch
import torch.nn as nn


class Layer(nn.Module):
    layer_name: str | None = None

    # ------------------------------------------------------------ reference API
    def backward(self, input: torch.Tensor, grad_output: torch.Tensor) -> torch.Tensor:
        """Gradient w.r.t. `input` given the gradient of the output; also
        accumulates parameter gradients into `.grad` (like the reference,
        which stores dweights/dbiases inside the layer)."""
        x = input.detach().requires_grad_(True)
        with torch.enable_grad():
            y = self.forward(x)
        params = [p for p in self.parameters() if p.requires_grad]
        grads = torch.autograd.grad(y, [x] + params, grad_output, allow_unused=True)
        for p, g in zip(params, grads[1:]):
            if g is None:
                continue
            if p.grad is None:
                p.grad = g.detach().clone()
            else:
                p.grad.add_(g)
        return grads[0]

    @torch.no_grad()
    def update(self, learning_rate: float) -> None:
        """Plain SGD step on the stored gradients (reference Layer::update)."""
        for p in self.parameters():
            if p.grad is not None:
                p.add_(p.grad, alpha=-learning_rate)

    def params(self) -> list[torch.Tensor]:
        return [p.detach() for p in self.parameters()]

    def gradients(self) -> list[torch.Tensor]:
        return [p.grad if p.grad is not None else torch.zeros_like(p) for p in self.parameters()]

    def set_gradients(self, grads) -> None:
        for p, g in zip(self.parameters(), grads):
            p.grad = g.clone()

    @torch.no_grad()
    def set_params(self, params) -> None:
        ps = list(self.parameters())
        if len(ps) != len(params):
            raise ValueError(f"{self.layer_type()} expects {len(ps)} parameter arrays, got {len(params)}")
        for p, v in zip(ps, params):
            p.copy_(torch.as_tensor(v, dtype=p.dtype, device=p.device).reshape(p.shape))

    # ParamLayer aliases
    get_parameters = params
    get_gradients = gradients
    set_parameters = set_params

    def set_training(self, training: bool) -> None:
        self.train(training)

    def is_training(self) -> bool:
        return self.training

    def layer_type(self) -> str:
        return type(self).__name__

    def parameter_count(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def layer_description(self) -> str:
        return f"type:{self.layer_type()}, params:{self.parameter_count()}"

    def name(self) -> str | None:
        return self.layer_name
