"""Pre-LN transformer block schedule shared by the fused engines (GPT, ViT).

One block, forward:  LN1 -> QKV gemm(+bias) -> flash attention -> proj gemm
(+bias +residual) -> LN2 -> fc1 gemm(+bias, GELU) -> fc2 gemm(+bias +residual).
Backward is the mirror image with the fused bias gradients (LayerNorm
backward column-sums its output = bias gradient of the projection that
wrote the residual stream; the dGELU epilogue column-sums dh = fc1 bias
gradient). Parameter names follow GPT-2 (`attn.c_attn`, `attn.c_proj`,
`mlp.c_fc`, `mlp.c_proj`, `ln_1`, `ln_2`) under a per-block prefix.

The encoder/decoder block of the reference (scirs2-neural/src/transformer/encoder.rs:21-700,
decoder.rs:22-470, models/architectures/gpt.rs block) computes the same
function on the CPU without a working backward.
"""
from __future__ import annotations

import torch

from ..ops import kernels as K
from ..utils.flat import FlatParams

BLOCK_PARAMS = [
    # name, shape(D, F), weight decay
    ("attn.c_attn.weight", lambda D, F: (3 * D, D), True),
    ("attn.c_proj.weight", lambda D, F: (D, D), True),
    ("mlp.c_fc.weight", lambda D, F: (F, D), True),
    ("mlp.c_proj.weight", lambda D, F: (D, F), True),
    ("attn.c_attn.bias", lambda D, F: (3 * D,), False),
    ("attn.c_proj.bias", lambda D, F: (D,), False),
    ("mlp.c_fc.bias", lambda D, F: (F,), False),
    ("mlp.c_proj.bias", lambda D, F: (D,), False),
    ("ln_1.weight", lambda D, F: (D,), False),
    ("ln_1.bias", lambda D, F: (D,), False),
    ("ln_2.weight", lambda D, F: (D,), False),
    ("ln_2.bias", lambda D, F: (D,), False),
]


def add_block_params(fp: FlatParams, prefix: str, D: int, F: int) -> None:
    for name, shape, decay in BLOCK_PARAMS:
        fp.add(prefix + name, shape(D, F), decay)


class BlockActs:
    """Preallocated activations of L blocks for a [B, S] micro-batch."""

    def __init__(self, L: int, B: int, S: int, D: int, F: int, H: int, device):
        M = B * S
        bf, f32 = torch.bfloat16, torch.float32
        e = lambda *s, dt=bf: torch.empty(*s, dtype=dt, device=device)  # noqa: E731
        self.B, self.S, self.M = B, S, M
        self.x = [e(M, D) for _ in range(L + 1)]  # residual stream entering block l
        self.ln1 = [e(M, D) for _ in range(L)]
        self.mu1 = [e(M, dt=f32) for _ in range(L)]
        self.rs1 = [e(M, dt=f32) for _ in range(L)]
        self.qkv = [e(M, 3 * D) for _ in range(L)]
        self.att = [e(M, D) for _ in range(L)]
        self.lse = [e(B, H, S, dt=f32) for _ in range(L)]
        self.xm = [e(M, D) for _ in range(L)]
        self.ln2 = [e(M, D) for _ in range(L)]
        self.mu2 = [e(M, dt=f32) for _ in range(L)]
        self.rs2 = [e(M, dt=f32) for _ in range(L)]
        self.h = [e(M, F) for _ in range(L)]
        self.g = [e(M, F) for _ in range(L)]
        # backward scratch (shared by all blocks)
        self.dres = e(M, D)
        self.dres2 = e(M, D)
        self.dln = e(M, D)
        self.datt = e(M, D)
        self.dqkv = e(M, 3 * D)
        self.dh = e(M, F)
        self.dq_acc = e(M * D, dt=f32)
        self.delta = e(B * H * S, dt=f32)
        self.ln_part = K.ln_partials(M, D, device)


def block_forward(fp: FlatParams, p: str, A: BlockActs, l: int, H: int, hd: int, eps: float, causal: bool) -> int:
    """Forward of block l (prefix p): A.x[l] -> A.x[l+1]. Returns kernel calls."""
    B, S = A.B, A.S
    K.layernorm_fwd(A.x[l], fp.w(p + "ln_1.weight"), fp.w(p + "ln_1.bias"), A.ln1[l], A.mu1[l], A.rs1[l], eps)
    K.gemm(A.ln1[l], fp.w(p + "attn.c_attn.weight"), A.qkv[l], bias=fp.w(p + "attn.c_attn.bias"))
    q, k, v = A.qkv[l].view(B, S, 3, H, hd).unbind(2)
    K.flash_attn_fwd(q, k, v, A.att[l].view(B, S, H, hd), A.lse[l], causal=causal)
    K.gemm(A.att[l], fp.w(p + "attn.c_proj.weight"), A.xm[l], epi=K.EPI_RESID, bias=fp.w(p + "attn.c_proj.bias"),
           aux=A.x[l])
    K.layernorm_fwd(A.xm[l], fp.w(p + "ln_2.weight"), fp.w(p + "ln_2.bias"), A.ln2[l], A.mu2[l], A.rs2[l], eps)
    K.gemm(A.ln2[l], fp.w(p + "mlp.c_fc.weight"), A.g[l], epi=K.EPI_BIAS_GELU, bias=fp.w(p + "mlp.c_fc.bias"),
           out2=A.h[l])
    K.gemm(A.g[l], fp.w(p + "mlp.c_proj.weight"), A.x[l + 1], epi=K.EPI_RESID, bias=fp.w(p + "mlp.c_proj.bias"),
           aux=A.xm[l])
    return 7


def block_backward(fp: FlatParams, p: str, A: BlockActs, l: int, H: int, hd: int, causal: bool,
                   prev_fc2_bias: str | None) -> int:
    """Backward of block l. On entry A.dres holds d loss / d x[l+1] (and the
    fc2 bias gradient colsum(dres) has already been accumulated by whoever
    produced dres); on exit A.dres holds d loss / d x[l] and, if
    `prev_fc2_bias` names the previous block's fc2 bias, its gradient
    colsum(d x[l]) has been accumulated."""
    B, S = A.B, A.S
    # fc2: x[l+1] = xm + g @ W2^T + b2 ; dh = (dres @ W2) * gelu'(h), colsum(dh) = fc1 bias grad
    K.gemm(A.dres, fp.w(p + "mlp.c_proj.weight"), A.dh, b_mn=True, epi=K.EPI_DGELU, aux=A.h[l],
           bias_grad=fp.g(p + "mlp.c_fc.bias"))
    K.gemm(A.dres, A.g[l], fp.g(p + "mlp.c_proj.weight"), a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
    # fc1: g = gelu(ln2 @ W1^T + b1)
    K.gemm(A.dh, fp.w(p + "mlp.c_fc.weight"), A.dln, b_mn=True)
    K.gemm(A.dh, A.ln2[l], fp.g(p + "mlp.c_fc.weight"), a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
    # ln2 (+ residual gradient); colsum(dres2) = attention proj bias gradient
    K.layernorm_bwd(A.dln, A.xm[l], fp.w(p + "ln_2.weight"), A.mu2[l], A.rs2[l], A.dres2, fp.g(p + "ln_2.weight"),
                    fp.g(p + "ln_2.bias"), A.ln_part, dresid=A.dres, dsum=fp.g(p + "attn.c_proj.bias"))
    # proj: xm = x + att @ Wp^T + bp
    K.gemm(A.dres2, fp.w(p + "attn.c_proj.weight"), A.datt, b_mn=True)
    K.gemm(A.dres2, A.att[l], fp.g(p + "attn.c_proj.weight"), a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
    # attention
    q, k, v = A.qkv[l].view(B, S, 3, H, hd).unbind(2)
    dq, dk, dv = A.dqkv.view(B, S, 3, H, hd).unbind(2)
    K.flash_attn_bwd(A.datt.view(B, S, H, hd), q, k, v, A.att[l].view(B, S, H, hd), A.lse[l], dq, dk, dv, A.dq_acc,
                     A.delta, causal=causal)
    # qkv
    K.gemm(A.dqkv, fp.w(p + "attn.c_attn.weight"), A.dln, b_mn=True)
    K.gemm(A.dqkv, A.ln1[l], fp.g(p + "attn.c_attn.weight"), a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
    K.bias_grad(A.dqkv, fp.g(p + "attn.c_attn.bias"))
    # ln1 (+ residual gradient) -> d x[l]
    K.layernorm_bwd(A.dln, A.x[l], fp.w(p + "ln_1.weight"), A.mu1[l], A.rs1[l], A.dres, fp.g(p + "ln_1.weight"),
                    fp.g(p + "ln_1.bias"), A.ln_part, dresid=A.dres2,
                    dsum=fp.g(prev_fc2_bias) if prev_fc2_bias else None)
    return 18


class FusedTrainerMixin:
    """Training-step plumbing shared by the fused engines: zero_grad, the
    fused AdamW configuration, gradient-sync hand-off and whole-step CUDA
    graph capture. The host class provides `fp` (FlatParams),
    `forward_backward(inputs, targets)`, `optimizer` and `grad_sync`."""

    kernel_launches = 0
    param_sync = None
    tracer = None  # utils.tracing.PhaseTimer: device time per phase of eager steps

    def _phase(self, name: str):
        import contextlib

        return self.tracer.phase(name) if self.tracer is not None else contextlib.nullcontext()

    def _params_begin(self):
        """Start the (ZeRO) parameter all-gather for this forward, if any."""
        if self.param_sync is not None:
            self.param_sync.begin_forward()

    def _wait_params(self, i: int):
        if self.param_sync is not None:
            self.param_sync.wait_bucket(i)

    def _params_end(self):
        if self.param_sync is not None:
            self.param_sync.end_forward()

    def zero_grad(self):
        self.fp.grad.zero_()

    def configure_adamw(self, lr=6e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_grad_norm=1.0):
        from ..optim.fused import FusedFlatOptimizer

        self.optimizer = FusedFlatOptimizer(
            self.fp, "adamw", lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, max_grad_norm=max_grad_norm
        )
        return self.optimizer

    def _train_step_eager(self, inputs: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        self.zero_grad()
        loss = self.forward_backward(inputs, targets)
        if self.grad_sync is not None:
            with self._phase("comm_wait"):
                self.grad_sync.finish()
        with self._phase("optimizer"):
            self.optimizer.step()
        self.kernel_launches += self.optimizer.launches_per_step
        return loss

    def enable_cuda_graph(self, enabled: bool = True):
        """Run the whole training step (forward, backward, gradient sync and
        the fused optimizer) as one captured CUDA graph. The first train_step
        at a given input shape runs eagerly (and initialises every buffer),
        the second captures and replays, later ones replay. Changing
        hyperparameters between steps is supported (they live in device
        memory); changing the input shape re-captures."""
        self.use_graph = enabled
        self._graph = None
        self._warm_key = None
        return self

    def release_cuda_graph(self):
        """Drop the captured graph (required before tearing down a process
        group whose collectives it captured)."""
        self._graph = None
        self._warm_key = None

    def _train_step_graphed(self, inputs, targets):
        key = (tuple(inputs.shape), inputs.dtype, tuple(targets.shape))
        if self._graph is not None and self._graph_key == key:
            self._g_in.copy_(inputs, non_blocking=True)
            self._g_tgt.copy_(targets, non_blocking=True)
            self._graph.replay()
            K.STATS.launches += self._graph_kernels
            if self.grad_sync is not None:
                self.grad_sync.launches += self._graph_comm
            self.optimizer.t += 1
            return self._g_loss
        if self._warm_key != key:
            self._warm_key = key
            return self._train_step_eager(inputs, targets)
        self._g_in = inputs.clone()
        self._g_tgt = targets.clone()
        torch.cuda.synchronize()
        k0 = K.STATS.launches
        c0 = self.grad_sync.launches if self.grad_sync is not None else 0
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._g_loss = self._train_step_eager(self._g_in, self._g_tgt)
        self._graph_kernels = K.STATS.launches - k0
        self._graph_comm = (self.grad_sync.launches - c0) if self.grad_sync is not None else 0
        K.STATS.launches = k0
        if self.grad_sync is not None:
            self.grad_sync.launches = c0
        self._graph, self._graph_key = g, key
        self.optimizer.t -= 1  # the capture did not execute a step; the replay below does
        return self._train_step_graphed(inputs, targets)

    def train_step(self, inputs: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """zero_grad -> forward/backward -> gradient sync -> fused optimizer step."""
        if self.optimizer is None:
            self.configure_adamw()
        if getattr(self, "use_graph", False) and inputs.is_cuda:
            return self._train_step_graphed(inputs, targets)
        return self._train_step_eager(inputs, targets)
