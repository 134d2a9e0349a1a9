"""MLP classifier (the reference's MNIST example network, scirs2-autograd/src/lib.rs:288
and benches/v030_neural_benchmarks.rs:78-442): Dense(784,128,relu) -> Dense(128,10),
softmax cross-entropy, Adam."""
from __future__ import annotations

import time

import torch

from ..nn.layers import Dense
from ..nn.losses import CrossEntropyLoss
from ..nn.sequential import Sequential


def mnist_mlp(hidden: int = 128, classes: int = 10, dtype=torch.float32, device=None, seed: int = 0) -> Sequential:
    return Sequential(
        Dense(784, hidden, "relu", seed=seed, dtype=dtype, device=device),
        Dense(hidden, classes, None, seed=seed + 1, dtype=dtype, device=device),
    )


def synthetic_mnist(n: int, seed: int = 0, device=None, dtype=torch.float32):
    """Inputs 28x28 uniform in [0, 1) and labels uniform in 0..9, seeded."""
    g = torch.Generator().manual_seed(seed)
    x = torch.rand(n, 784, generator=g, dtype=torch.float32).to(dtype)
    y = torch.randint(0, 10, (n,), generator=g)
    return x.to(device), y.to(device)


def train_mnist_mlp(steps: int = 100, batch: int = 64, lr: float = 1e-3, seed: int = 0, device=None,
                    dtype=torch.float32, checkpoint_path: str | None = None) -> dict:
    """Runs the MLP configuration and returns timing and the loss curve."""
    from ..training.serialization import save_model

    model = mnist_mlp(dtype=dtype, device=device, seed=seed)
    model.compile(optimizer="adam", loss=CrossEntropyLoss(), learning_rate=lr)
    x, y = synthetic_mnist(steps * batch, seed=seed, device=device, dtype=dtype)
    losses = []
    model.train_batch(x[:batch], y[:batch])  # builds the fused optimizer state
    model2 = mnist_mlp(dtype=dtype, device=device, seed=seed)
    model.load_state_dict(model2.state_dict())
    model.optimizer = None
    model._ensure_opt()
    t0 = time.perf_counter()
    for i in range(steps):
        losses.append(model.train_batch(x[i * batch : (i + 1) * batch], y[i * batch : (i + 1) * batch]))
    dt = time.perf_counter() - t0
    if checkpoint_path:
        save_model(model, checkpoint_path)
    return {"steps": steps, "seconds": dt, "steps_per_s": steps / dt, "losses": losses, "model": model}
