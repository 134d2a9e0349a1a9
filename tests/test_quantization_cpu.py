"""Quantization formats and methods (CPU)."""
import torch
import torch.nn as nn

from scirs_b200 import quantization as Q


def test_int8_roundtrip_and_matmul():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(16, 32, generator=g)
    for mode in Q.Int8Mode:
        for gran in Q.Granularity:
            q = Q.quantize_int8(x, mode, gran)
            assert q.data.dtype == torch.int8 and q.shape == (16, 32)
            err = (Q.dequantize_int8(q) - x).abs().max()
            step = float(q.scale.max())
            assert err <= 0.51 * step + 1e-6, (mode, gran, float(err), step)
    assert Q.roundtrip_mse(x, Q.Int8Mode.SYMMETRIC, Q.Granularity.PER_CHANNEL) <= Q.roundtrip_mse(x)
    a, b = torch.randn(8, 64, generator=g), torch.randn(64, 5, generator=g)
    assert torch.allclose(Q.quantized_matmul(a, b), a @ b, atol=0.25)


def test_int4_pack_and_groups():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(3, 70, generator=g)
    q = Q.quantize_int4(x, Q.GroupSize.G32)
    assert q.packed.numel() == (210 + 1) // 2 and q.scale.numel() == 7
    assert q.compression_ratio() > 4
    d = Q.dequantize_int4(q)
    assert d.shape == x.shape
    assert float((d - x).abs().max()) <= 0.51 * float(q.scale.max()) + 1e-6
    # low nibble holds the even element
    q2 = Q.quantize_int4(torch.tensor([0.0, 15.0]), 32)
    assert int(q2.packed[0]) & 0xF == 0 and int(q2.packed[0]) >> 4 == 15


def test_gptq_beats_rounding_on_correlated_inputs():
    g = torch.Generator().manual_seed(2)
    base = torch.randn(512, 16, generator=g)
    x = base @ torch.randn(16, 64, generator=g) + 0.05 * torch.randn(512, 64, generator=g)
    w = torch.randn(32, 64, generator=g)
    res = Q.GptqQuantizer(Q.GptqConfig(bits=3, group_size=32, block_size=16)).quantize_with_calibration(w, x)
    naive = Q.naive_quantize(w, 3, 32)
    e_gptq = float(((x @ res.quantized_weights.t() - x @ w.t()) ** 2).mean())
    e_naive = float(((x @ naive.t() - x @ w.t()) ** 2).mean())
    assert e_gptq < 0.8 * e_naive, (e_gptq, e_naive)


def test_awq_and_smoothquant():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(256, 64, generator=g)
    x[:, :4] *= 30.0  # outlier channels
    w = torch.randn(16, 64, generator=g)
    layer = Q.AwqQuantizer(Q.AwqConfig(bits=4, group_size=32, search_steps=10)).quantize(w, x)
    e_awq = float(((layer.forward(x) - x @ w.t()) ** 2).mean())
    e_naive = float(((x @ Q.naive_quantize(w, 4, 32).t() - x @ w.t()) ** 2).mean())
    assert e_awq <= e_naive * 1.0001
    xs, ws, s = Q.smooth_linear(x, w, 0.5)
    assert torch.allclose(xs @ ws.t(), x @ w.t(), rtol=1e-4, atol=1e-3)
    assert float(xs.abs().amax(0).max() / xs.abs().amax(0).min()) < float(x.abs().amax(0).max() / x.abs().amax(0).min())


def test_observers_ptq_and_qat():
    r = Q.minmax_calibration_runner()
    for i in range(3):
        r.observe("a", torch.linspace(-i - 1, i + 1, 11))
    assert r.get_stats("a").max_val == 3.0
    p = Q.PercentileObserver(90.0)
    p.observe(torch.arange(100.0))
    st = p.stats()
    assert 85 < st.max_val < 95 and 5 < st.min_val < 15
    m = Q.MovingAverageObserver(0.5)
    m.observe(torch.tensor([0.0, 2.0]))
    m.observe(torch.tensor([0.0, 4.0]))
    assert m.stats().max_val == 3.0
    ptq = Q.PostTrainingQuantizer(Q.QuantizationConfig(bits=8))
    ptq.add_calibration_data("w", torch.tensor([-2.0, 1.0]))
    params = ptq.finalize_calibration()
    assert abs(params["w"].scale - 2.0 / 127) < 1e-9
    net = nn.Sequential(nn.Linear(8, 16), nn.ReLU(), nn.Linear(16, 1))
    Q.QuantizationAwareTraining(8).prepare(net)
    assert isinstance(net[0], Q.FakeQuantLinear)
    opt = torch.optim.SGD(net.parameters(), lr=0.05)
    gen = torch.Generator().manual_seed(4)
    xb = torch.randn(64, 8, generator=gen)
    yb = xb.sum(1, keepdim=True)
    l0 = None
    for _ in range(60):
        loss = ((net(xb) - yb) ** 2).mean()
        l0 = l0 if l0 is not None else float(loss)
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert float(loss) < 0.3 * l0
