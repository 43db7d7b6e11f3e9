"""Launcher: layer order, --set parsing, env validation, torchrun command."""

import pytest

from vllm_cmp170hx_b200.launch import main as launch

SETTINGS = __import__("pathlib").Path(__file__).resolve().parent.parent / "examples" / "settings" / "config3"


def test_layers_and_set():
    cfg, files = launch.resolve(SETTINGS, "tp4", ["nccl"], ["engine.max-num-seqs=96", "env.VLLM_B200_KV_PLAN_LOG=true"])
    assert cfg["model"] == "config3"
    assert cfg["engine"]["max-num-seqs"] == 96  # --set beats the layout (128) and defaults (64)
    assert cfg["engine"]["max-model-len"] == 4096  # model layer beats defaults
    assert cfg["env"]["VLLM_B200_ALLREDUCE"] == "nccl"  # overlay beats model
    argv, env = launch.command(cfg)
    assert "torch.distributed.run" in argv and "--nproc-per-node=4" in argv
    assert argv[argv.index("--max-num-seqs") + 1] == "96" and env["VLLM_B200_KV_PLAN_LOG"] == "True"


def test_rejects_retired_and_unknown_env():
    with pytest.raises(launch.LaunchError):
        launch.resolve(SETTINGS, "tp1", [], ["env.VLLM_AMPERE_DECODE_KERNELS=1"])
    with pytest.raises(launch.LaunchError):
        launch.resolve(SETTINGS, "tp1", [], ["env.VLLM_B200_NOT_A_FLAG=1"])


def test_receipt_hashes_inputs(tmp_path):
    cfg, files = launch.resolve(SETTINGS, "tp1")
    argv, env = launch.command(cfg)
    rec = launch.receipt(cfg, files, argv, env)
    assert len(rec["inputs"]) == 3 and all(len(h) == 64 for h in rec["inputs"].values())


def test_dflash_overlay_reaches_the_server_command():
    from vllm_cmp170hx_b200.api.server import engine_config, parse_args

    cfg, _files = launch.resolve(SETTINGS, "tp1", ["dflash"], ["engine.device=\"cpu\""])
    argv, _env = launch.command(cfg)
    server = argv[argv.index("vllm_cmp170hx_b200.api.server") + 1:]
    sc = engine_config(parse_args(server)).scheduler
    assert (sc.num_speculative_tokens, sc.spec_method, sc.adaptive_k) == (3, "dflash", "by_load")
