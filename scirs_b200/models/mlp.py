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


def numpy_reference_losses(W1, b1, W2, b2, x, y, steps, batch, lr, b1_=0.9, b2_=0.999, eps=1e-8):
    """Loss curve of the same configuration in float64 NumPy, written from the
    reference's math (scirs2-neural/src/layers/dense.rs:174-420 Dense y = xW + b
    with W [in, out]; losses/crossentropy.rs:54-143 mean softmax cross-entropy;
    optimizers/adam.rs:163-215 bias-corrected Adam): the CPU oracle of the MLP
    configuration, since the reference itself cannot be built here."""
    import numpy as np

    P = [W1.copy(), b1.copy(), W2.copy(), b2.copy()]
    m = [np.zeros_like(p) for p in P]
    v = [np.zeros_like(p) for p in P]
    out = []
    for t in range(1, steps + 1):
        xb, yb = x[(t - 1) * batch : t * batch], y[(t - 1) * batch : t * batch]
        h = xb @ P[0] + P[1]
        a = np.maximum(h, 0)
        z = a @ P[2] + P[3]
        z = z - z.max(1, keepdims=True)
        p = np.exp(z) / np.exp(z).sum(1, keepdims=True)
        out.append(float(-np.log(p[np.arange(batch), yb]).mean()))
        dz = p.copy()
        dz[np.arange(batch), yb] -= 1
        dz /= batch
        G = [None] * 4
        G[2], G[3] = a.T @ dz, dz.sum(0)
        dh = (dz @ P[2].T) * (h > 0)
        G[0], G[1] = xb.T @ dh, dh.sum(0)
        for i in range(4):
            m[i] = b1_ * m[i] + (1 - b1_) * G[i]
            v[i] = b2_ * v[i] + (1 - b2_) * G[i] ** 2
            P[i] = P[i] - lr * (m[i] / (1 - b1_**t)) / (np.sqrt(v[i] / (1 - b2_**t)) + eps)
    return out


def main():
    """MLP 784-128-10 configuration on the CPU: 100 Adam steps at batch 64 in
    fp32, steps/s, the loss curve against the float64 oracle, and the
    mnist_model.json round trip. Prints one JSON line."""
    import argparse
    import json
    import os
    import tempfile

    from ..training.serialization import load_model

    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--threads", type=int, default=0)
    a = ap.parse_args()
    if a.threads:
        torch.set_num_threads(a.threads)
    init = mnist_mlp(seed=0)
    ws = [t.detach().double().numpy() for t in
          (init.layers()[0].weight, init.layers()[0].bias, init.layers()[1].weight, init.layers()[1].bias)]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "mnist_model.json")
        r = train_mnist_mlp(steps=a.steps, batch=a.batch, lr=1e-3, seed=0, checkpoint_path=path)
        x, y = synthetic_mnist(a.steps * a.batch, seed=0)
        ref = numpy_reference_losses(*ws, x.double().numpy(), y.numpy(), a.steps, a.batch, 1e-3)
        m2 = load_model(path, dtype=torch.float32)
        probe = torch.rand(8, 784, generator=torch.Generator().manual_seed(1))
        r["model"].eval()
        same = bool(torch.allclose(m2(probe), r["model"](probe)))
        size = os.path.getsize(path)
    L = r["losses"]
    print(json.dumps({
        "config": "MLP 784-128-10 ReLU, softmax cross-entropy, fp32 CPU, Adam lr 1e-3, batch 64",
        "data": "synthetic: inputs uniform [0,1) from seed 0, labels uniform in 0..9",
        "steps": a.steps, "seconds": round(r["seconds"], 4), "steps_per_s": round(r["steps_per_s"], 1),
        "threads": torch.get_num_threads(),
        "loss_every_10": [round(L[i], 5) for i in range(0, a.steps, 10)] + [round(L[-1], 5)],
        "max_abs_diff_vs_float64_oracle": max(abs(p - q) for p, q in zip(L, ref)),
        "checkpoint": {"format": "mnist_model.json", "bytes": size, "reload_matches": same},
    }))


if __name__ == "__main__":
    main()
