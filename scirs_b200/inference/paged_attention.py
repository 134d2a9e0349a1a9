"""Single-query (decode) attention over paged KV caches.

:class:`PagedAttentionForward` computes, for every active sequence, the
attention of its newest query ([H, HD]) over the sequence's whole page chain,
with grouped-query heads (H query heads over Hkv cached heads). On the GPU
this is the split-key decode kernel of scirs_b200/csrc/paged_attention.cu
(bandwidth-bound: each cached K/V byte is read once per sequence and KV head)
followed by a combine kernel; on the CPU a PyTorch restatement.

Reference parity: scirs2-neural/src/inference/paged_attention.rs:37-283
(PagedAttentionConfig, PagedAttentionForward::forward(query, page_chain,
pool)).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _ext
from .kv_cache import BlockManager, InferenceError, KvPagePool


@dataclass
class PagedAttentionConfig:
    num_heads: int = 8
    head_dim: int = 64
    scale: float | None = None
    tokens_per_split: int = 512


class PagedAttentionForward:
    def __init__(self, config: PagedAttentionConfig):
        self.config = config
        self._scratch = {}

    def _scale(self):
        c = self.config
        return c.scale if c.scale is not None else c.head_dim ** -0.5

    def forward(self, query: torch.Tensor, page_chain: list[int], pool: KvPagePool, seq_len: int | None = None):
        """One sequence: query [H, HD], its page chain, and (optionally) its
        length in tokens (default: the whole chain)."""
        bs = pool.config.block_size
        n = seq_len if seq_len is not None else len(page_chain) * bs
        if query.shape != (self.config.num_heads, self.config.head_dim):
            raise InferenceError("query shape does not match the configuration")
        bt = torch.tensor([page_chain], dtype=torch.int32, device=pool.device)
        lens = torch.tensor([n], dtype=torch.int32, device=pool.device)
        return self.forward_batch(query.reshape(1, *query.shape), pool, bt, lens)[0]

    def forward_batch(self, q: torch.Tensor, pool: KvPagePool, block_tables: torch.Tensor, seq_lens: torch.Tensor):
        """q [B, H, HD]; block_tables [B, max_pages] int32; seq_lens [B] int32."""
        B, H, HD = q.shape
        if q.is_cuda:
            c = self.config
            span = block_tables.shape[1] * pool.config.block_size
            splits = max(1, (span + c.tokens_per_split - 1) // c.tokens_per_split)
            key = (B, H, HD, splits)
            if key not in self._scratch:
                self._scratch = {key: (torch.empty(B, H, splits, HD, device=q.device),
                                       torch.empty(B, H, splits, 2, device=q.device))}
            po, pml = self._scratch[key]
            out = torch.empty(B, H, HD, dtype=torch.bfloat16, device=q.device)
            _ext.kernels().paged_attention_decode(q.to(torch.bfloat16).contiguous(), pool.k, pool.v,
                                                  block_tables.contiguous(), seq_lens.contiguous(), out, po, pml,
                                                  c.tokens_per_split, self._scale())
            return out
        return paged_attention_reference(q, pool, block_tables, seq_lens, self._scale())

    def forward_manager(self, q: torch.Tensor, manager: BlockManager, seq_ids: list[int]):
        """Decode attention for the given sequences of a BlockManager."""
        manager.sync()
        rows = torch.tensor([manager.row_of(s) for s in seq_ids], dtype=torch.long, device=manager.block_tables.device)
        return self.forward_batch(q, manager.pool, manager.block_tables[rows].contiguous(),
                                  manager.seq_lens[rows].contiguous())


def paged_attention_reference(q, pool: KvPagePool, block_tables, seq_lens, scale):
    """fp32 PyTorch restatement (oracle)."""
    B, H, HD = q.shape
    Hkv = pool.config.num_heads
    G = H // Hkv
    bs = pool.config.block_size
    out = torch.empty(B, H, HD, dtype=torch.bfloat16, device=q.device)
    for b in range(B):
        n = int(seq_lens[b])
        pages = block_tables[b, : (n + bs - 1) // bs].long().to(pool.k.device)
        k = pool.k[pages].reshape(-1, Hkv, HD)[:n].float()
        v = pool.v[pages].reshape(-1, Hkv, HD)[:n].float()
        k = k.repeat_interleave(G, dim=1)
        v = v.repeat_interleave(G, dim=1)
        s = torch.einsum("hd,thd->ht", q[b].float(), k) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("ht,thd->hd", p, v).to(torch.bfloat16)
    return out
