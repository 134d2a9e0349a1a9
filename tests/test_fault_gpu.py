"""Device-side failure detection: a bounded wait on a peer flag that nothing
sets gives up after its timeout, records the error in the device status
word and returns; the host turns it into an exception and the CUDA context
stays usable."""
import pytest
import torch

from scirs_b200 import _ext

pytestmark = pytest.mark.gpu


def test_peer_wait_timeout_reports_status_and_context_survives():
    dev = torch.device("cuda", 0)
    _ext.check_status(0)
    rows, Vl, world = 16, 64, 2
    logits = torch.randn(rows, Vl, device=dev).bfloat16()
    tgt = torch.randint(0, Vl, (rows,), device=dev)
    stats = torch.zeros(world, rows, 4, device=dev)
    loss = torch.zeros(rows, device=dev)
    flags = torch.zeros(8, dtype=torch.int32, device=dev)  # rank 1 never signals
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    _ext.kernels().tp_xent_finish(logits, tgt, stats, loss, Vl * world, 0, 0, 1.0, flags, epoch, 1, 0.05)
    ev1.record()
    torch.cuda.synchronize()
    waited_ms = ev0.elapsed_time(ev1)
    assert 40.0 <= waited_ms < 5000.0, waited_ms
    with pytest.raises(RuntimeError, match="peer wait timed out"):
        _ext.check_status(0)
    _ext.check_status(0)  # cleared by the read
    # the context still works: the same kernel with nothing to wait on
    _ext.kernels().tp_xent_finish(logits, tgt, stats, loss, Vl * world, 0, 0, 1.0, flags, epoch, 0, 0.05)
    x = torch.ones(1 << 20, device=dev)
    assert float(x.sum()) == float(1 << 20)
    torch.cuda.synchronize()
    _ext.check_status(0)


def test_out_of_range_token_is_reported_not_faulted():
    dev = torch.device("cuda", 0)
    _ext.check_status(0)
    V, D, S = 100, 64, 4
    wte = torch.randn(V, D, device=dev).bfloat16()
    tok = torch.tensor([[1, 2, V + 5, 3]], device=dev)  # one id past the vocabulary
    out = torch.zeros(4, D, device=dev, dtype=torch.bfloat16)
    _ext.kernels().embedding_fwd(tok.reshape(-1), wte, None, out, S)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="bounds check failed"):
        _ext.check_status(0)
    torch.testing.assert_close(out[0].float(), wte[1].float())
    assert float(out[2].float().abs().sum()) == 0.0  # the bad row was skipped
