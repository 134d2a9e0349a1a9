"""Encoder-decoder transformer on the kernels (bf16, cross-attention with a
different source length) against the same model in fp32 through PyTorch:
loss and gradients."""
import copy

import pytest
import torch

from scirs_b200.models.seq2seq import Transformer, TransformerConfig
from scirs_b200.ops import kernels as K

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("act,norm_first", [("relu", False), ("gelu", True)])
def test_seq2seq_kernels_match_fp32(act, norm_first, monkeypatch):
    cfg = TransformerConfig(d_model=256, n_encoder_layers=2, n_decoder_layers=2, n_heads=4, d_ff=1024,
                            max_seq_len=512, src_vocab=512, tgt_vocab=640, activation=act, norm_first=norm_first)
    ref = Transformer(cfg, seed=5)
    m = copy.deepcopy(ref).cuda().bfloat16()
    ref = ref.cuda()
    with torch.no_grad():  # the fp32 copy holds the same bf16-rounded weights
        for p, q in zip(ref.parameters(), m.parameters()):
            p.copy_(q.float())
    g = torch.Generator().manual_seed(0)
    src = torch.randint(0, 512, (4, 300), generator=g).cuda()
    tgt = torch.randint(0, 640, (4, 129), generator=g).cuda()
    k0 = K.STATS.launches
    loss = m.loss(src, tgt[:, :-1], tgt[:, 1:])
    loss.backward()
    assert K.STATS.launches - k0 > 50  # GEMM / attention / LayerNorm / CE kernels ran
    monkeypatch.setenv("SCIRS_KERNELS", "torch")
    lref = ref.loss(src, tgt[:, :-1], tgt[:, 1:])
    lref.backward()
    assert abs(float(loss) - float(lref)) < 3e-2, (float(loss), float(lref))
    for (n, p), q in zip(m.named_parameters(), ref.parameters()):
        if q.grad is None or q.grad.norm() == 0:
            continue
        err = float((p.grad.float() - q.grad).norm() / q.grad.norm())
        assert err < 6e-2, (n, err)
