"""Sequential model with the reference's Keras-like training API.

  scirs2-neural/src/models/sequential.rs:15-360 (fit / train_batch /
  predict / predict_batched / evaluate), scirs2-neural/src/layers/mod.rs:137-300
  (add / len / total_parameters / layer_info), and the Python contract of
  scirs2-python/tests/test_neural.py:8-50,305-352 (compile / is_compiled /
  train_step / evaluate).

Unlike the reference (whose Sequential::train_batch silently never applies
the optimizer to concrete layers, sequential.rs:305-336), every parameter is
updated here: the optimizer is one of the fused flat-buffer optimizers.
"""
from __future__ import annotations

import math

import torch

from ..optim.optimizers import get_optimizer
from ..training.history import History, TrainingConfig
from .base import Layer
from .losses import get_loss


class Sequential(Layer):
    def __init__(self, *layers):
        super().__init__()
        self.layers_ = torch.nn.ModuleList(layers)
        self.loss_fn = None
        self.optimizer = None
        self.history = History()

    # ------------------------------------------------------------ structure
    def add(self, layer):
        self.layers_.append(layer)
        self.optimizer = None  # parameters changed; rebuild on next compile/step
        return self

    def __len__(self):
        return len(self.layers_)

    def num_layers(self) -> int:
        return len(self.layers_)

    def layers(self):
        return list(self.layers_)

    def total_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def layer_info(self) -> list[str]:
        out = []
        for i, l in enumerate(self.layers_):
            desc = l.layer_description() if isinstance(l, Layer) else type(l).__name__
            out.append(f"Layer {i}: {desc}")
        return out

    def summary(self) -> str:
        return "\n".join(self.layer_info() + [f"Total parameters: {self.total_parameters()}"])

    def forward(self, x):
        for l in self.layers_:
            x = l(x)
        return x

    # ------------------------------------------------------------ training
    def compile(self, optimizer="adam", loss="mse", learning_rate: float | None = None, **opt_kwargs):
        self.loss_fn = get_loss(loss)
        self._opt_spec = (optimizer, learning_rate, opt_kwargs)
        self.optimizer = get_optimizer(optimizer, self.parameters(), learning_rate, **opt_kwargs) if isinstance(
            optimizer, str) else optimizer
        return self

    def is_compiled(self) -> bool:
        return self.loss_fn is not None

    def _ensure_opt(self):
        if self.optimizer is None:
            if not self.is_compiled():
                raise RuntimeError("call compile(optimizer=..., loss=...) first")
            o, lr, kw = self._opt_spec
            self.optimizer = get_optimizer(o, self.parameters(), lr, **kw)

    def train_batch(self, x, y) -> float:
        """One optimizer step on a batch; returns the batch loss."""
        self._ensure_opt()
        self.train()
        self.optimizer.zero_grad()
        loss = self.loss_fn(self(x), y)
        loss.backward()
        for cb in getattr(self, "_pre_step_callbacks", ()):
            cb.on_before_step(self)  # e.g. gradient clipping
        self.optimizer.step()
        return float(loss.detach())

    train_step = train_batch

    @torch.no_grad()
    def predict(self, x):
        self.eval()
        return self(x)

    @torch.no_grad()
    def predict_batched(self, x, batch_size: int = 256):
        self.eval()
        return torch.cat([self(x[i : i + batch_size]) for i in range(0, x.shape[0], batch_size)])

    @torch.no_grad()
    def evaluate(self, x, y, batch_size: int | None = None) -> float:
        if self.loss_fn is None:
            raise RuntimeError("compile the model first")
        self.eval()
        if batch_size is None:
            return float(self.loss_fn(self(x), y))
        tot, n = 0.0, 0
        for i in range(0, x.shape[0], batch_size):
            xb, yb = x[i : i + batch_size], y[i : i + batch_size]
            tot += float(self.loss_fn(self(xb), yb)) * xb.shape[0]
            n += xb.shape[0]
        return tot / max(n, 1)

    def fit(self, x, y, epochs: int = 10, batch_size: int = 32, validation_split: float = 0.0, shuffle: bool = True,
            callbacks=None, verbose: int = 0, config: TrainingConfig | None = None, seed: int = 0) -> History:
        """Mini-batch training with an optional trailing validation split
        (the split is taken from the end of the data, as the reference does)."""
        if config is not None:
            epochs, batch_size = config.epochs, config.batch_size
            validation_split, shuffle, verbose = config.validation_split, config.shuffle, config.verbose
        n = x.shape[0]
        split = int((1.0 - validation_split) * n) if validation_split > 0 else n
        xt, yt = x[:split], y[:split]
        xv, yv = (x[split:], y[split:]) if split < n else (None, None)
        cbs = callbacks or []
        self._pre_step_callbacks = [cb for cb in cbs if hasattr(cb, "on_before_step")]
        g = torch.Generator().manual_seed(seed)
        for cb in cbs:
            cb.on_train_begin(self)
        for ep in range(epochs):
            for cb in cbs:
                cb.on_epoch_begin(ep, self)
            idx = torch.randperm(split, generator=g) if shuffle else torch.arange(split)
            idx = idx.to(xt.device)
            tot, cnt = 0.0, 0
            for b in range(math.ceil(split / batch_size)):
                sel = idx[b * batch_size : (b + 1) * batch_size]
                l = self.train_batch(xt[sel], yt[sel])
                tot += l * sel.numel()
                cnt += sel.numel()
                for cb in cbs:
                    cb.on_batch_end(b, self, {"loss": l})
            logs = {"loss": tot / max(cnt, 1)}
            self.history.train_loss.append(logs["loss"])
            if xv is not None and xv.shape[0] > 0:
                logs["val_loss"] = self.evaluate(xv, yv)
                self.history.val_loss.append(logs["val_loss"])
            if verbose:
                print(f"epoch {ep + 1}/{epochs} " + " ".join(f"{k}={v:.5f}" for k, v in logs.items()))
            stop = False
            for cb in cbs:
                cb.on_epoch_end(ep, self, logs)
                stop = stop or cb.stop_training
            if stop:
                break
        for cb in cbs:
            cb.on_train_end(self)
        self._pre_step_callbacks = []
        return self.history
