"""Paged KV cache bookkeeping, paged decode attention (reference path),
speculative decoding and cached generation on the CPU."""
import torch

from scirs_b200.inference import (BlockManager, BlockManagerConfig, GPTGenerator, KvPageConfig, KvPagePool,
                                  PagedAttentionConfig, PagedAttentionForward, SharedPrefixCache,
                                  SpeculativeConfig, SpeculativeDecoder, TokenDist, Xorshift64)
from scirs_b200.models.gpt import GPTConfig, GPTModel


def test_block_manager_chains_and_append():
    pool = KvPagePool(8, KvPageConfig(block_size=4, num_heads=2, head_dim=8), "cpu")
    bm = BlockManager(pool, BlockManagerConfig(max_sequences=3, max_pages_per_seq=4))
    bm.allocate_sequence(7)
    bm.allocate_sequence(9)
    k = torch.randn(10, 2, 8).to(torch.bfloat16)
    v = torch.randn(10, 2, 8).to(torch.bfloat16)
    bm.append([7, 9], [6, 4], k, v)
    assert bm.seq_len(7) == 6 and len(bm.sequence_page_chain(7)) == 2
    assert bm.seq_len(9) == 4 and len(bm.sequence_page_chain(9)) == 1
    p1 = bm.sequence_page_chain(7)[1]
    assert torch.equal(pool.k[p1, 1], k[5])
    free = pool.free_count()
    bm.free_sequence(7)
    assert pool.free_count() == free + 2 and bm.active_sequences() == 1
    c = SharedPrefixCache()
    h = SharedPrefixCache.compute_prefix_hash([1, 2, 3])
    c.insert(h, [4, 5])
    assert c.lookup(h) == [4, 5] and len(c) == 1 and c.evict(h) == [4, 5] and c.is_empty()


def test_paged_attention_matches_dense():
    torch.manual_seed(0)
    H, Hkv, hd, bs = 8, 2, 16, 4
    pool = KvPagePool(16, KvPageConfig(block_size=bs, num_heads=Hkv, head_dim=hd), "cpu")
    bm = BlockManager(pool, BlockManagerConfig(max_sequences=2, max_pages_per_seq=8))
    bm.allocate_sequence(0)
    n = 11
    k = torch.randn(n, Hkv, hd).to(torch.bfloat16)
    v = torch.randn(n, Hkv, hd).to(torch.bfloat16)
    bm.append([0], [n], k, v)
    q = torch.randn(1, H, hd).to(torch.bfloat16)
    out = PagedAttentionForward(PagedAttentionConfig(H, hd)).forward_manager(q, bm, [0])
    kk = k.float().repeat_interleave(H // Hkv, 1)
    vv = v.float().repeat_interleave(H // Hkv, 1)
    p = torch.softmax(torch.einsum("hd,thd->ht", q[0].float(), kk) * hd**-0.5, -1)
    ref = torch.einsum("ht,thd->hd", p, vv)
    assert torch.allclose(out[0].float(), ref, atol=2e-2)


def test_speculative_identical_models_accept_everything():
    d = TokenDist([1.0, 2.0, 3.0])
    assert abs(float(d.softmax().sum()) - 1.0) < 1e-12
    lg = [0.0] * 8
    pre, tok = SpeculativeDecoder.rejection_sampling_step([lg, lg], [lg, lg], [0, 1], SpeculativeConfig(top_p=1.0))
    assert pre == [0, 1] and 0 <= tok < 8
    rng = Xorshift64(3)
    assert 0.0 <= rng.next_f64() < 1.0

    vocab = 16
    g = torch.Generator().manual_seed(0)
    tlog = torch.randn(vocab, generator=g)

    def draft(ctx):
        return [(int(torch.argmax(tlog)), tlog.tolist()) for _ in range(3)]

    def target(ctx, toks):
        return [tlog.tolist() for _ in toks]

    res = SpeculativeDecoder.decode([1, 2], draft, target, SpeculativeConfig(max_tokens=9, top_p=1.0))
    assert len(res.accepted_tokens) == 9 and res.acceptance_rate == 1.0


def test_speculative_preserves_target_distribution():
    """Draft uniform, target peaked: the sampled first tokens follow the target."""
    vocab = 4
    target = torch.tensor([2.0, 0.0, 0.0, -1.0])
    cfg = SpeculativeConfig(top_p=1.0, temperature=1.0)
    rng = Xorshift64(11)
    counts = torch.zeros(vocab)
    for i in range(4000):
        x = int(rng.next_u64() % vocab)  # draft sample from the uniform draft
        pre, tok = SpeculativeDecoder.rejection_sampling_step([[0.0] * vocab], [target.tolist()], [x], cfg, rng)
        counts[pre[0] if pre else tok] += 1
    emp = counts / counts.sum()
    assert torch.allclose(emp, torch.softmax(target, 0), atol=0.03), emp


def test_cached_generation_matches_recompute_cpu():
    cfg = GPTConfig.tiny(vocab=128, seq=64)
    m = GPTModel(cfg, device="cpu", seed=1)
    gen = GPTGenerator(m, max_sequences=2, max_len=64, block_size=8)
    prompt = torch.randint(0, cfg.vocab_size, (10,), generator=torch.Generator().manual_seed(3))
    out = gen.generate([prompt], max_new_tokens=6)[0]
    seq = prompt.tolist()
    ref = []
    for _ in range(6):
        lg = m.logits(torch.tensor([seq]))
        t = int(torch.argmax(lg[0, -1].float()))
        ref.append(t)
        seq.append(t)
    assert out == ref, (out, ref)
