"""Index layout of the expert-parallel peer kernels, emulated on CPU.

The dispatch kernel stores send row q = (w * L + l) * C + c of source rank s
into rank w's buffer at row l * (W * C) + s * C + c; the combine kernel reads
token t's assignment (e, slot) from rank e // L at row
((e % L) * W + s) * C + slot. This test restates both formulas in torch,
drives them with the layer's own routing and send-row map, and checks the
result against the single-device mixture of experts on each rank's tokens.
"""
import torch

from scirs_b200.nn.moe import MixtureOfExperts, MoEConfig, _send_rows, route


def _emulate(ref: MixtureOfExperts, xs, W):
    E = ref.config.num_experts
    L = E // W
    d = xs[0].shape[1]
    routings, idxs = [], []
    for x in xs:
        r = route(ref.gate_logits(x), ref.config)
        q, tok, _ = _send_rows(r, E, x.shape[0])
        idx = torch.full((E * r.capacity,), -1, dtype=torch.long)
        idx[q] = tok
        routings.append(r)
        idxs.append(idx)
    C = routings[0].capacity
    # dispatch: every source writes into every owner's [L * W * C, d] buffer
    recv = [torch.zeros(L * W * C, d) for _ in range(W)]
    for s in range(W):
        for qrow in range(W * L * C):
            w, rem = divmod(qrow, L * C)
            l, c = divmod(rem, C)
            t = int(idxs[s][qrow])
            recv[w][l * (W * C) + s * C + c] = xs[s][t] if t >= 0 else 0.0
    # experts on each owner (its slice of the stacked weights)
    ys = []
    for w in range(W):
        e = ref.experts
        sl = slice(w * L, (w + 1) * L)
        h = torch.relu(torch.baddbmm(e.b1[sl, None, :], recv[w].view(L, W * C, d), e.w1[sl]))
        ys.append(torch.baddbmm(e.b2[sl, None, :], h, e.w2[sl]).reshape(L * W * C, d))
    # combine: each source reads its tokens' outputs from the owners
    outs = []
    for s, (x, r) in enumerate(zip(xs, routings)):
        out = torch.zeros_like(x)
        T, k = r.expert.shape
        for t in range(T):
            for j in range(k):
                slot = int(r.slot[t, j])
                if slot < 0:
                    continue
                e = int(r.expert[t, j])
                out[t] += r.weight[t, j] * ys[e // L][((e % L) * W + s) * C + slot]
        outs.append(out)
    return outs


def test_peer_kernel_layout_matches_single_device():
    torch.manual_seed(0)
    W = 2
    cfg = MoEConfig(num_experts=4, expert_dim=16, top_k=2, capacity_factor=1.0)
    ref = MixtureOfExperts(8, cfg, seed=7)
    xs = [torch.randn(12, 8) for _ in range(W)]
    with torch.no_grad():
        outs = _emulate(ref, xs, W)
        for x, o in zip(xs, outs):
            assert torch.allclose(o, ref(x), atol=1e-5, rtol=1e-5)
