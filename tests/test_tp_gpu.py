"""Tensor-parallel decoder engine at TP=1 vs the fp32 PyTorch oracle (rotary
positions, untied LM head, vocabulary-parallel cross-entropy code path)."""
import socket

import pytest
import torch
import torch.distributed as dist

from scirs_b200 import _ext
from scirs_b200.models.torch_gpt import TorchDecoder
from scirs_b200.models.tp_gpt import DecoderConfig, TPDecoder
from scirs_b200.parallel.tensor_parallel import TPContext

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture
def pg():
    store = dist.TCPStore("127.0.0.1", _port(), 1, True)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, device_id=torch.device("cuda", 0))
    yield
    dist.destroy_process_group()


def test_tp_decoder_matches_oracle_gpu(pg):
    cfg = DecoderConfig.tiny(vocab=1024, seq=256)
    B, S = 4, 256
    dev = torch.device("cuda", 0)
    ctx = TPContext(TPDecoder.heap_bytes(cfg, B, S, 1))
    m = TPDecoder(cfg, ctx, batch=B, seq=S, seed=2)
    # bf16-round the master weights so both sides start from identical values
    m.fp.master.copy_(m.fp.master.to(torch.bfloat16).float())
    m.fp.sync_bf16()
    ref = TorchDecoder(cfg, seq=S).to(dev)
    ref.load_full((n, m.fp.m(n).detach()) for n in m.fp.order)
    g = torch.Generator().manual_seed(0)
    t = torch.randint(0, cfg.vocab_size, (B, S + 1), generator=g).to(dev)
    x, y = t[:, :-1].contiguous(), t[:, 1:].contiguous()
    m.zero_grad()
    loss = m.forward_backward(x, y)
    lref = ref(x, y)
    lref.backward()
    torch.cuda.synchronize()
    _ext.check_status(0)
    assert abs(float(loss) - float(lref)) < 3e-2, (float(loss), float(lref))
    grads = ref.full_grads()
    for name in m.fp.order:
        gr, mine = grads[name], m.fp.g(name)
        if name.endswith("c_attn.bias"):
            D = cfg.hidden_size  # the key bias has an exactly-zero gradient
            mine, gr = torch.cat([mine[:D], mine[2 * D :]]), torch.cat([gr[:D], gr[2 * D :]])
        err = float((mine - gr).norm() / (gr.norm() + 1e-8))
        assert err < 6e-2, (name, err)
    m.close()
    ctx.close()


def test_tp_decoder_trains_gpu(pg):
    cfg = DecoderConfig.tiny(vocab=1024, seq=256)
    B, S = 4, 256
    dev = torch.device("cuda", 0)
    ctx = TPContext(TPDecoder.heap_bytes(cfg, B, S, 1))
    m = TPDecoder(cfg, ctx, batch=B, seq=S, seed=0)
    m.configure_adamw(lr=2e-3, weight_decay=0.0)
    m.enable_cuda_graph()
    g = torch.Generator().manual_seed(2)
    t = torch.randint(0, cfg.vocab_size, (B, S + 1), generator=g).to(dev)
    x, y = t[:, :-1].contiguous(), t[:, 1:].contiguous()
    l0 = float(m.train_step(x, y))
    for _ in range(25):
        loss = float(m.train_step(x, y))
    _ext.check_status(0)
    assert loss < l0 - 1.0, (l0, loss)
    m.close()
    ctx.close()
