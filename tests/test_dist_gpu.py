"""Multi-GPU tests: in-kernel NVLink collectives and data-parallel training.

Each test launches tests/dist_worker.py with torchrun as child processes
(NCCL's NVLS disabled, short process-group timeout, hard `timeout` around it)
and checks rank 0's JSON verdict. Every case runs at 2, 4 and 8 ranks; a
size is skipped when fewer GPUs are visible.
"""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


NPROC = [2, 4, 8]


def _run(case, tmp_path, nproc=2, port=29611):
    port += 40 * {2: 0, 4: 1, 8: 2}.get(nproc, 3)
    if torch.cuda.device_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    out = tmp_path / f"{case}.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(HERE, "dist_worker.py"), case, str(out)]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    return json.load(open(out))


@pytest.mark.parametrize("nproc", NPROC)
def test_nvlink_collectives(tmp_path, nproc):
    res = _run("collectives", tmp_path, nproc=nproc, port=29611)
    for k, v in res.items():
        if k.startswith("allreduce"):
            assert v["identical"], k
            assert v["max_err"] < 2e-2, (k, v)
        elif k.startswith("reduce_scatter"):
            assert v["max_err"] < 2e-2, (k, v)
        else:
            assert v["equal"], k


@pytest.mark.parametrize("nproc", NPROC)
def test_nvls_allreduce(tmp_path, nproc):
    res = _run("nvls", tmp_path, nproc=nproc, port=29615)
    if "skipped" in res:
        pytest.skip(res["skipped"])
    for k, v in res.items():
        assert v["identical"], k
        tol = 1e-5 if "float32" in k else 2e-2
        assert v["max_err"] < tol, (k, v)


@pytest.mark.parametrize("nproc", NPROC)
def test_ring_attention(tmp_path, nproc):
    res = _run("ring_attn", tmp_path, nproc=nproc, port=29616)
    for k, v in res.items():
        for name in ("o", "dq", "dk", "dv"):
            assert v[name] < 2e-2, (k, name, v)
        assert v["lse"] < 2e-2, (k, v)


@pytest.mark.parametrize("nproc", NPROC)
def test_data_parallel_gpt(tmp_path, nproc):
    res = _run("dp_gpt", tmp_path, nproc=nproc, port=29612)
    ref = res["single"]["losses"]
    for mode in ("fused", "nccl"):
        assert res[mode]["replica_max_diff"] == 0.0, mode
        for a, b in zip(res[mode]["losses"], ref):
            assert abs(a - b) < 2e-2, (mode, res[mode]["losses"], ref)


@pytest.mark.parametrize("nproc", NPROC)
def test_zero_vit(tmp_path, nproc):
    res = _run("zero_vit", tmp_path, nproc=nproc, port=29613)
    ref = res["single"]["losses"]
    for mode in ("fused", "nccl"):
        for a, b in zip(res[mode]["losses"], ref):
            assert abs(a - b) < 3e-2, (mode, res[mode]["losses"], ref)


@pytest.mark.parametrize("nproc", NPROC)
def test_tensor_parallel_decoder(tmp_path, nproc):
    res = _run("tp_decoder", tmp_path, nproc=nproc, port=29614)
    ref = res["single"]["losses"]
    for mode in ("fused", "nccl"):
        for a, b in zip(res[mode]["losses"], ref):
            assert abs(a - b) < 3e-2, (mode, res[mode]["losses"], ref)


@pytest.mark.parametrize("nproc", NPROC)
def test_expert_parallel_peer_kernels(tmp_path, nproc):
    res = _run("ep_moe", tmp_path, nproc=nproc, port=29617)
    for it, v in res.items():
        for name, err in v.items():
            assert err < 3e-2, (it, name, v)


@pytest.mark.parametrize("nproc", NPROC)
def test_pipeline_parallel_gpt(tmp_path, nproc):
    res = _run("pp_gpt", tmp_path, nproc=nproc, port=29618)
    ref = res["single"]["losses"]
    for sched in ("1f1b", "gpipe", "1f1b_graph"):
        assert res[sched]["tied_diff"] == 0.0, (sched, res[sched])
        for a, b in zip(res[sched]["losses"], ref):
            assert abs(a - b) < 2e-2, (sched, res[sched]["losses"], ref)


@pytest.mark.parametrize("nproc", NPROC)
def test_zero_gpt(tmp_path, nproc):
    res = _run("zero_gpt", tmp_path, nproc=nproc, port=29619)
    ref = res["single"]["losses"]
    assert res["fused"]["early_vocab"], res["fused"]
    for mode in ("fused", "nccl"):
        assert res[mode]["replica_max_diff"] == 0.0, mode
        for a, b in zip(res[mode]["losses"], ref):
            assert abs(a - b) < 2e-2, (mode, res[mode]["losses"], ref)
