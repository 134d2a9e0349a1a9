"""Encoder-decoder transformer: causality of the decoder, dependence on the
source through cross-attention, pre-/post-LN variants, training reduces the
loss (CPU: the reference semantics of every op)."""
import torch

from scirs_b200.models.seq2seq import Transformer, TransformerConfig


def _cfg(**kw):
    base = dict(d_model=64, n_encoder_layers=2, n_decoder_layers=2, n_heads=2, d_ff=128, max_seq_len=64,
                src_vocab=40, tgt_vocab=48)
    base.update(kw)
    return TransformerConfig(**base)


def test_decoder_is_causal_and_uses_the_source():
    m = Transformer(_cfg(), seed=1)
    g = torch.Generator().manual_seed(0)
    src = torch.randint(0, 40, (2, 11), generator=g)
    tgt = torch.randint(0, 48, (2, 9), generator=g)
    a = m.logits(src, tgt)
    tgt2 = tgt.clone()
    tgt2[:, 6:] = (tgt2[:, 6:] + 1) % 48
    b = m.logits(src, tgt2)
    assert torch.allclose(a[:, :6], b[:, :6], atol=1e-5) and not torch.allclose(a[:, 6:], b[:, 6:])
    src2 = src.clone()
    src2[:, -1] = (src2[:, -1] + 1) % 40
    c = m.logits(src2, tgt)
    assert not torch.allclose(a[:, 0], c[:, 0])  # every target position sees the whole source


def test_features_api_and_pre_ln():
    m = Transformer(_cfg(norm_first=True, src_vocab=0, tgt_vocab=0, pos_encoding_type="learned"), seed=2)
    src, tgt = torch.randn(3, 10, 64), torch.randn(3, 7, 64)
    out = m.forward_train(src, tgt)
    assert out.shape == (3, 7, 64)
    assert torch.allclose(m.forward_inference(src, tgt), out)


def test_training_reduces_loss():
    torch.manual_seed(0)
    m = Transformer(_cfg(), seed=3)
    opt = torch.optim.Adam(m.parameters(), lr=3e-3)
    g = torch.Generator().manual_seed(1)
    src = torch.randint(0, 40, (8, 12), generator=g)
    tgt = (src[:, :10] + 1) % 48  # learnable mapping
    first = None
    for _ in range(60):
        opt.zero_grad()
        loss = m.loss(src, tgt[:, :-1], tgt[:, 1:])
        loss.backward()
        opt.step()
        first = float(loss) if first is None else first
    assert float(loss) < 0.5 * first
