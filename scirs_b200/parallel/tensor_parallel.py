"""Tensor parallelism (Megatron-style, sequence-parallel) on fused
communication + GEMM kernels.

Activations between the column- and row-parallel layers are split over the
ranks by tokens (rank r holds rows [r*Mr, (r+1)*Mr) of the M = world*Mr
tokens). The four communication points of a block become:

  all-gather -> GEMM  (QKV, FC1 forward; proj/FC2 data gradients): every
      rank keeps a full-size gathered buffer in its symmetric heap. The
      producer writes its rows into its own buffer, then the copy engines
      push those rows into every peer's buffer at the same offset and, on
      the same copy stream, write the step's flag value into each peer's
      flag word (no SM involved, so a peer whose SMs are all busy in a GEMM
      still receives data and flags). The GEMM reads only local memory: its
      TMA producer starts with this rank's own rows and waits (bounded) on a
      peer's flag only before its first tile of that peer's rows, so the
      transfer overlaps the MMAs, and every row crosses NVLink exactly once.
  GEMM -> reduce-scatter  (proj, FC2 forward; QKV/FC1 data gradients):
      the epilogue pushes each output row's bf16 partial sums into the
      owner's receive slot over NVLink as soon as the tile is done; the last
      CTA signals; the owner sums the world slots (+ bias + residual) in one
      pass.
  weight gradients read the gathered buffers locally.

Mode "nccl" runs the same schedule with torch.distributed all_gather /
reduce_scatter and separate GEMMs: the unfused baseline.

Reference parity: scirs2-neural/src/training/tensor_parallel.rs:85-385
(ColumnParallelLinear / RowParallelLinear / vocabulary-partitioned layers as
single-process slices).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _ext
from ..ops import kernels as K
from .symmetric import SymmetricHeap


class TPContext:
    def __init__(self, heap_bytes: int, mode: str = "fused", timeout_s: float = 10.0, group=None):
        assert mode in ("fused", "nccl")
        self.mode = mode
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.timeout_s = float(timeout_s)
        self.heap = SymmetricHeap(heap_bytes, group=group) if mode == "fused" else None
        if self.heap is not None:
            # Two flag arrays (one word per source rank): row 0 is written by
            # the copy engines (gathers, in copy-stream order), row 1 by
            # kernels (reduce-scatter / statistics, in main-stream order), so
            # each word only ever increases.
            fl = self.heap.alloc((2, 8), torch.int32, align=256)
            self.flags_ce, self.flags = fl[0], fl[1]
            self.sig_ce = [a + 4 * self.rank for a in self.heap.peer_addrs(self.flags_ce)]
            self.sig = [a + 4 * self.rank for a in self.heap.peer_addrs(self.flags)]
        else:
            self.flags = self.flags_ce = None
            self.sig, self.sig_ce = [], []
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.vals = torch.zeros(4096, dtype=torch.int32, device=self.device)  # this step's flag values
        self.copy_stream = torch.cuda.Stream(self.device) if mode == "fused" else None
        self._copied = False
        self.idx = 0
        self._recv = None
        self._recv_i = 0
        self.launches = 0

    # ------------------------------------------------------------- buffers
    def alloc(self, shape, dtype=torch.bfloat16) -> torch.Tensor:
        """A buffer peers can read (heap in fused mode, plain otherwise)."""
        if self.heap is not None:
            return self.heap.alloc(shape, dtype)
        return torch.empty(*shape, dtype=dtype, device=self.device)

    def recv_buffers(self, rows: int, D: int):
        """Two alternating receive buffers [world, rows, D] for GEMM->RS. A
        rank reuses a buffer only two reductions later, after every peer has
        consumed the one in between, so two suffice."""
        if self._recv is None:
            if self.heap is not None:
                self._recv = [self.heap.alloc((self.world, rows, D)) for _ in range(2)]
            else:
                self._recv = [torch.empty(self.world, rows, D, dtype=torch.bfloat16, device=self.device)
                              for _ in range(2)]
        assert self._recv[0].shape[1] == rows and self._recv[0].shape[2] == D, "one receive shape per context"
        r = self._recv[self._recv_i]
        self._recv_i ^= 1
        return r

    # ------------------------------------------------------------- signals
    def begin_step(self):
        _ext.kernels().tp_step_begin(self.epoch, self.vals)
        self.idx = 0
        self._recv_i = 0

    def finish(self):
        """Join the copy stream (before anything outside the step reads or
        reuses buffers the copies touch)."""
        if self.copy_stream is not None and self._copied:
            torch.cuda.current_stream(self.device).wait_stream(self.copy_stream)
            self._copied = False

    def segment(self, full: torch.Tensor) -> torch.Tensor:
        """This rank's rows of a gathered [M, ...] buffer."""
        n = full.shape[0] // self.world
        return full[self.rank * n : (self.rank + 1) * n]

    def gather(self, full: torch.Tensor) -> int:
        """All-gather the rows of `full` (this rank's segment is written):
        fused -> copy-engine pushes + flag words, returns the signal id the
        consumer waits on; nccl -> in-place all_gather, returns 0."""
        seg = self.segment(full)
        if self.mode != "fused":
            if self.world > 1:
                dist.all_gather_into_tensor(full, seg, group=self.group)
            return 0
        i = self._next()
        if self.world > 1:
            main = torch.cuda.current_stream(self.device)
            self.copy_stream.wait_stream(main)
            self._copied = True
            with torch.cuda.stream(self.copy_stream):
                comm = _ext.comm()
                comm.peer_copy(self.heap.peer_addrs(seg), seg.data_ptr(), seg.numel() * seg.element_size())
                comm.peer_copy(self.sig_ce, self.vals.data_ptr() + 4 * i, 4)
        self.launches += 1
        return i

    def _next(self) -> int:
        self.idx += 1
        return self.idx

    def publish(self) -> int:
        """Signal that everything this rank wrote so far (on this stream) is
        visible to the peers. Returns the signal id consumers wait on."""
        if self.mode != "fused":
            return 0
        i = self._next()
        _ext.kernels().tp_signal(self.sig, self.epoch, i)
        self.launches += 1
        return i

    # ------------------------------------------------------------- GEMMs
    def ag_gemm(self, full, ready: int, b, out, *, b_mn=False, epi=K.EPI_BF16, bias=None, aux=None, out2=None,
                rope=None):
        """out[M, N] = full[M, K] @ op(b), where `full` is a gathered buffer
        whose peer segments arrive after signal `ready` (see :meth:`gather`).
        epi=EPI_ROPE with rope=(cos, sin, S, hd, cols) applies the rotary
        embedding in the epilogue."""
        if self.mode == "fused" and self.world > 1:
            seg = self.segment(full)
            step = seg.numel() * seg.element_size()
            addrs = [full.data_ptr() + r * step for r in range(self.world)]
            rc, rsn, rS, rhd, rcols = rope if rope is not None else (None, None, 0, 0, 0)
            _ext.kernels().gemm_tp(seg, b, out, 0, int(b_mn), int(epi), bias, aux, out2, False, 0, self.rank,
                                   self.world, addrs, [], [], self.flags_ce, self.epoch, ready, [], 0,
                                   self.timeout_s, rc, rsn, int(rS), int(rhd), int(rcols))
        else:
            K.gemm(full, b, out, b_mn=b_mn, epi=epi, bias=bias, aux=aux, out2=out2, rope=rope)
        self.launches += 1
        return out

    def gemm_rs(self, a, b, rows: int, *, b_mn=False, partial=None):
        """Partial products a @ op(b) of all M rows, reduce-scattered by rows:
        returns (recv buffer, signal id) for :meth:`reduce`. In nccl mode
        `partial` ([M, N] bf16) is the local product buffer."""
        N = b.shape[1] if b_mn else b.shape[0]
        recv = self.recv_buffers(rows, N)
        if self.mode == "fused":
            i = self._next()
            _ext.kernels().gemm_tp(a, b, recv, 0, int(b_mn), K.EPI_BF16, None, None, None, False, 0, self.rank,
                                   self.world, [], [], self.heap.peer_addrs(recv[self.rank]), None, self.epoch, 0,
                                   self.sig, i, self.timeout_s)
            self.launches += 1
            return recv, i
        K.gemm(a, b, partial, b_mn=b_mn)
        dist.reduce_scatter_tensor(recv[0], partial, group=self.group)
        return recv, 0

    def reduce(self, recv, sig: int, out, bias=None, resid=None):
        """out = resid + bias + sum of the receive slots."""
        if self.mode == "fused":
            _ext.kernels().tp_reduce(recv, out, bias, resid, self.rank, self.flags, self.epoch, sig, [], 0,
                                     self.timeout_s)
        else:
            _ext.kernels().tp_reduce(recv[:1], out, bias, resid, 0, None, self.epoch, 0, [], 0, self.timeout_s)
        self.launches += 1
        return out

    def wgrad(self, a, b, out):
        """out[M', N] += a^T b over all tokens (both [tokens, .]; gathered
        operands are local full-size buffers)."""
        K.gemm(a, b, out, a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
        self.launches += 1
        return out

    def close(self):
        if self.heap is not None:
            self.heap.close()
            self.heap = None
