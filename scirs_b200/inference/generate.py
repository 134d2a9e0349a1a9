"""Cached autoregressive generation for the GPT engine.

Prefill runs the engine's own forward over each prompt (flash attention) and
appends every layer's keys/values into a paged cache; each decode step then
processes one new token per active sequence: embedding -> per layer
LayerNorm -> QKV GEMM -> append K/V (paged_kv_append) -> paged decode
attention over the sequence's page chain -> projection GEMM (+residual) ->
LayerNorm -> GELU MLP GEMMs -> final LayerNorm -> LM head -> next token.
All layers share one page table (the pages of layer l live in layer l's
pool at the same page ids).

Reference parity: the reference generates with its (placeholder) GPT on the
CPU without a cache (scirs2-neural/src/models/architectures/gpt.rs); the
page management follows scirs2-neural/src/inference/block_manager.rs.
"""
from __future__ import annotations

import torch

from .. import _ext
from ..ops import kernels as K
from .kv_cache import BlockManager, BlockManagerConfig, KvPageConfig, KvPagePool
from .paged_attention import PagedAttentionConfig, PagedAttentionForward


class GPTGenerator:
    def __init__(self, model, max_sequences: int = 16, max_len: int | None = None, block_size: int = 16,
                 num_pages: int | None = None):
        self.m = model
        cfg = model.cfg
        self.cfg = cfg
        self.L, self.H, self.hd, self.D = cfg.num_hidden_layers, cfg.num_attention_heads, cfg.head_dim, cfg.hidden_size
        max_len = max_len or cfg.max_position_embeddings
        pages_per_seq = (max_len + block_size - 1) // block_size
        num_pages = num_pages or max_sequences * pages_per_seq
        pc = KvPageConfig(block_size=block_size, num_heads=self.H, head_dim=self.hd)
        self.pools = [KvPagePool(num_pages, pc, model.device) for _ in range(self.L)]
        self.manager = BlockManager(self.pools[0], BlockManagerConfig(max_sequences, pages_per_seq))
        self.attn = PagedAttentionForward(PagedAttentionConfig(self.H, self.hd))
        self.max_len = max_len
        self._next_id = 0
        self.last_token: dict[int, int] = {}

    # ----------------------------------------------------------- helpers
    def _append(self, l: int, rows, pos, k, v):
        dev = self.m.device
        mgr = self.manager
        if k.is_cuda:
            r = torch.tensor(rows, dtype=torch.int32).to(dev, non_blocking=True)
            p = torch.tensor(pos, dtype=torch.int32).to(dev, non_blocking=True)
            _ext.kernels().paged_kv_append(k.contiguous(), v.contiguous(), self.pools[l].k, self.pools[l].v,
                                           mgr.block_tables, r, p)
        else:
            bs = self.pools[0].config.block_size
            for i, (row, ps) in enumerate(zip(rows, pos)):
                pid = int(mgr._bt_host[row, ps // bs])
                self.pools[l].k[pid, ps % bs] = k[i]
                self.pools[l].v[pid, ps % bs] = v[i]

    # ----------------------------------------------------------- API
    @torch.no_grad()
    def add_sequence(self, prompt: torch.Tensor) -> int:
        """Prefill one prompt (1-D token tensor); returns the sequence id."""
        m, H, hd = self.m, self.H, self.hd
        S = int(prompt.numel())
        assert 0 < S < self.max_len
        sid = self._next_id
        self._next_id += 1
        self.manager.allocate_sequence(sid)
        rows, pos = self.manager.reserve([sid], [S])
        self.manager.sync()
        tok = prompt.to(m.device).reshape(1, S)
        logits = m.logits(tok)  # runs every layer; keeps qkv per layer in the activations
        A = m._acts
        for l in range(self.L):
            qkv = A.qkv[l].view(S, 3, H, hd)
            self._append(l, rows, pos, qkv[:, 1], qkv[:, 2])
        nxt = int(torch.argmax(logits[0, -1].float()))
        self.last_token[sid] = nxt
        return sid

    @torch.no_grad()
    def step(self, seq_ids: list[int], temperature: float = 0.0, generator=None) -> list[int]:
        """Feed each sequence's pending token, return the next tokens."""
        m, fp, cfg = self.m, self.m.fp, self.cfg
        H, hd, D = self.H, self.hd, self.D
        n = len(seq_ids)
        dev = m.device
        toks = torch.tensor([self.last_token[s] for s in seq_ids], dtype=torch.long, device=dev)
        lens = [self.manager.seq_len(s) for s in seq_ids]
        posn = torch.tensor(lens, dtype=torch.long, device=dev)
        rows, pos = self.manager.reserve(seq_ids, [1] * n)
        self.manager.sync()
        bf, f32 = torch.bfloat16, torch.float32
        x = (fp.w("wte")[toks].float() + fp.w("wpe")[posn].float()).to(bf).contiguous()
        ln = torch.empty(n, D, dtype=bf, device=dev)
        mu, rs = torch.empty(n, dtype=f32, device=dev), torch.empty(n, dtype=f32, device=dev)
        qkv = torch.empty(n, 3 * D, dtype=bf, device=dev)
        xm = torch.empty(n, D, dtype=bf, device=dev)
        h = torch.empty(n, cfg.intermediate_size, dtype=bf, device=dev)
        g = torch.empty(n, cfg.intermediate_size, dtype=bf, device=dev)
        idx = torch.tensor([self.manager.row_of(s) for s in seq_ids], dtype=torch.long, device=dev)
        bt = self.manager.block_tables[idx].contiguous()
        sl = self.manager.seq_lens[idx].contiguous()
        eps = cfg.layer_norm_eps
        for l in range(self.L):
            p = f"h{l}."
            K.layernorm_fwd(x, fp.w(p + "ln_1.weight"), fp.w(p + "ln_1.bias"), ln, mu, rs, eps)
            K.gemm(ln, fp.w(p + "attn.c_attn.weight"), qkv, bias=fp.w(p + "attn.c_attn.bias"))
            q3 = qkv.view(n, 3, H, hd)
            self._append(l, rows, pos, q3[:, 1], q3[:, 2])
            att = self.attn.forward_batch(q3[:, 0].contiguous(), self.pools[l], bt, sl)
            K.gemm(att.view(n, D), fp.w(p + "attn.c_proj.weight"), xm, epi=K.EPI_RESID,
                   bias=fp.w(p + "attn.c_proj.bias"), aux=x)
            K.layernorm_fwd(xm, fp.w(p + "ln_2.weight"), fp.w(p + "ln_2.bias"), ln, mu, rs, eps)
            K.gemm(ln, fp.w(p + "mlp.c_fc.weight"), g, epi=K.EPI_BIAS_GELU, bias=fp.w(p + "mlp.c_fc.bias"), out2=h)
            x2 = torch.empty_like(x)
            K.gemm(g, fp.w(p + "mlp.c_proj.weight"), x2, epi=K.EPI_RESID, bias=fp.w(p + "mlp.c_proj.bias"), aux=xm)
            x = x2
        K.layernorm_fwd(x, fp.w("ln_f.weight"), fp.w("ln_f.bias"), ln, mu, rs, eps)
        logits = torch.empty(n, cfg.vocab_padded, dtype=bf, device=dev)
        K.gemm(ln, fp.w("wte"), logits)
        lg = logits[:, : cfg.vocab_size].float()
        if temperature > 0:
            nxt = torch.multinomial(torch.softmax(lg / temperature, -1), 1, generator=generator).view(-1)
        else:
            nxt = torch.argmax(lg, dim=-1)
        out = [int(t) for t in nxt.tolist()]
        for s, t in zip(seq_ids, out):
            self.last_token[s] = t
        return out

    def generate(self, prompts: list[torch.Tensor], max_new_tokens: int, temperature: float = 0.0) -> list[list[int]]:
        """Greedy (temperature 0) or sampled continuation of every prompt."""
        ids = [self.add_sequence(p) for p in prompts]
        outs = {s: [self.last_token[s]] for s in ids}
        for _ in range(max_new_tokens - 1):
            for s, t in zip(ids, self.step(ids, temperature)):
                outs[s].append(t)
        for s in ids:
            self.release(s)
        return [outs[s] for s in ids]

    def release(self, seq_id: int):
        self.manager.free_sequence(seq_id)
        self.last_token.pop(seq_id, None)
