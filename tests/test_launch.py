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


def test_checkpoint_manifest_verify_and_stamp(tmp_path):
    """A manifest of a checkpoint directory verifies; a changed byte is a mismatch, a truncated file or a
    missing shard is incomplete, a missing directory absent; a verified check leaves a stamp whose
    unchanged files are not hashed again."""
    import json

    from vllm_cmp170hx_b200.launch import provenance as pv

    ck = tmp_path / "ck"
    ck.mkdir()
    (ck / "config.json").write_text(json.dumps({"model_type": "x"}))
    (ck / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"a": "s1.safetensors",
                                                                               "b": "s2.safetensors"}}))
    (ck / "s1.safetensors").write_bytes(b"1" * 100)
    (ck / "s2.safetensors").write_bytes(b"2" * 50)
    man = pv.checkpoint_manifest(ck)
    assert sorted(man["files"]) == ["config.json", "model.safetensors.index.json", "s1.safetensors", "s2.safetensors"]
    stamp = tmp_path / "stamp.json"
    assert pv.verify_checkpoint(ck, man, stamp) == ("verified", {})
    assert json.loads(stamp.read_text())["schema"] == pv.STAMP_SCHEMA
    calls = []
    orig = pv.sha256_file
    pv.sha256_file = lambda p, *a: calls.append(p) or orig(p)
    try:
        assert pv.verify_checkpoint(ck, man, stamp)[0] == "verified"
        assert calls == []  # every identity matched the stamp
    finally:
        pv.sha256_file = orig
    (ck / "s1.safetensors").write_bytes(b"1" * 99 + b"x")
    st, probs = pv.verify_checkpoint(ck, man, stamp)
    assert st == "mismatch" and list(probs) == ["s1.safetensors"]
    (ck / "s2.safetensors").write_bytes(b"2" * 10)
    assert pv.verify_checkpoint(ck, man)[0] == "incomplete"
    (ck / "s2.safetensors").unlink()
    assert pv.verify_checkpoint(ck, man)[0] == "incomplete"
    assert pv.verify_checkpoint(tmp_path / "nope", man)[0] == "absent"
    assert pv.main(["verify", "--path", str(tmp_path / "nope"), "--manifest", str(_write(tmp_path, man))]) == 6


def _write(tmp_path, man):
    import json

    p = tmp_path / "man.json"
    p.write_text(json.dumps(man))
    return p


def test_receipt_records_tree_native_and_checkpoint(tmp_path):
    from vllm_cmp170hx_b200.launch import main as launch
    from vllm_cmp170hx_b200.launch import provenance as pv

    tree = pv.tree_state()
    assert set(tree) >= {"commit", "dirty", "changed"}
    nat = pv.native_identity()
    assert "path" in nat
    cfg = {"model": "config3"}
    rec = launch.receipt(cfg, [], ["x"], {}, {"path": "p", "manifest_sha256": "0" * 64, "status": "verified"})
    assert rec["tree"]["commit"] == tree["commit"] and rec["checkpoint"]["status"] == "verified"
    # a checkpoint that does not verify refuses the launch
    ck = tmp_path / "ck"
    ck.mkdir()
    (ck / "config.json").write_text("{}")
    man = pv.checkpoint_manifest(ck)
    (ck / "config.json").write_text("{ }")
    try:
        launch.check_launch({"model": str(ck)}, False, _write(tmp_path, man))
        raise AssertionError("expected a refusal")
    except launch.LaunchError as e:
        assert "incomplete" in str(e) or "mismatch" in str(e)
