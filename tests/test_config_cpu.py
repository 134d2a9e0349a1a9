"""Run configuration: the packaged benchmark configs load and validate,
SCIRS_* environment variables override them, unknown keys are rejected."""
import pytest

from scirs_b200 import config as C


def test_packaged_configs_load():
    names = C.list_configs()
    assert {"mlp_mnist_cpu", "gpt2_small_dp", "vit_b16_zero", "decoder_1p3b_tp8", "kernel_sweep"} <= set(names)
    g = C.load_config("gpt2_small_dp", env={})
    assert g.model == "gpt2" and g.data.global_batch == 64 and g.data.seq_len == 1024
    assert g.parallel.dp == 8 and g.parallel.zero == 1
    g.parallel.validate(world=8)
    mc = g.model_config()
    assert mc.hidden_size == 768 and mc.num_hidden_layers == 12 and mc.vocab_size == 50257
    t = C.load_config("decoder_1p3b_tp8", env={})
    assert t.parallel.tp == 8 and t.model_config().hidden_size == 2048
    m = C.load_config("mlp_mnist_cpu", env={})
    assert m.optim.name == "adam" and m.runtime.steps == 100


def test_env_overrides():
    env = {"SCIRS_PARALLEL_DP": "4", "SCIRS_DATA_GLOBAL_BATCH": "32", "SCIRS_COMM": "nccl",
           "SCIRS_WAIT_TIMEOUT_S": "2.5", "SCIRS_OPTIM_BETAS": "0.8,0.9", "SCIRS_RUNTIME_CUDA_GRAPH": "0"}
    g = C.load_config("gpt2_small_dp", env=env)
    assert g.parallel.dp == 4 and g.data.global_batch == 32
    assert g.parallel.dp_mode == "nccl" and g.runtime.wait_timeout_s == 2.5
    assert g.optim.betas == (0.8, 0.9) and g.runtime.cuda_graph is False
    with pytest.raises(ValueError):
        g.parallel.validate(world=8)


def test_rejects_unknown_keys_and_bad_layouts(tmp_path):
    p = tmp_path / "bad.json"
    p.write_text('{"model": "gpt2", "parallel": {"dpp": 2}}')
    with pytest.raises(KeyError):
        C.load_config(str(p), env={})
    with pytest.raises(ValueError):
        C.ParallelConfig(pp=4, micro_batches=2).validate()
    assert C.ParallelConfig(dp=2, tp=4).world_size == 8
    assert C.ParallelConfig(dp=2, tp=4).describe() == "dp2+tp4"
