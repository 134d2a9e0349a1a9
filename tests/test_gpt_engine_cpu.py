"""The hand-scheduled GPT forward/backward (run on the CPU reference paths of
every op) must match PyTorch autograd on the same weights."""
import torch

from scirs_b200.models.gpt import GPTConfig, GPTModel
from scirs_b200.models.torch_gpt import TorchGPT


def _cfg():
    c = GPTConfig.tiny(vocab=200, seq=32)
    c.hidden_size, c.num_attention_heads, c.intermediate_size, c.num_hidden_layers = 128, 2, 256, 2
    return c


def test_engine_matches_autograd_cpu():
    torch.manual_seed(0)
    cfg = _cfg()
    m = GPTModel(cfg, device="cpu", seed=3)
    # bf16 storage: compare against an fp32 oracle holding the same bf16-rounded weights
    sd = {k: v.to(torch.bfloat16).float() for k, v in m.state_dict().items()}
    m.load_state_dict(sd)
    ref = TorchGPT(cfg)
    ref.load_flat_state(sd)
    tok = torch.randint(0, cfg.vocab_size, (2, 33))
    x, y = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
    m.zero_grad()
    loss = m.forward_backward(x, y)
    lref = ref(x, y)
    lref.backward()
    assert abs(float(loss) - float(lref)) < 2e-2
    grads = ref.flat_grads()
    for name, g in grads.items():
        mine = m.fp.g(name)
        if name == "wte":
            mine = mine[: cfg.vocab_size]
        err = float((mine - g).norm() / (g.norm() + 1e-8))
        assert err < 5e-2, (name, err)


def test_engine_training_reduces_loss_cpu():
    cfg = _cfg()
    m = GPTModel(cfg, device="cpu", seed=0)
    m.configure_adamw(lr=3e-3, weight_decay=0.0)
    g = torch.Generator().manual_seed(1)
    tok = torch.randint(0, cfg.vocab_size, (4, 33), generator=g)
    x, y = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
    l0 = float(m.train_step(x, y))
    for _ in range(15):
        l = float(m.train_step(x, y))
    assert l < l0 - 0.5
