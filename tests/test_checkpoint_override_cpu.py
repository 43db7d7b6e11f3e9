"""Override sidecars (the reference's override-sidecar/2, kernels/exl3/override.py): a plain tensor
the export stored at lower precision is restored from the sidecar after every check, and each
failing check refuses before anything is replaced; read-ahead of the shards."""

import json
import os

import pytest
import torch
from safetensors.torch import save_file

from vllm_cmp170hx_b200 import hf_loader
from vllm_cmp170hx_b200.checkpoint_override import Readahead, apply_override, build_override


def _export(tmp_path):
    g = torch.Generator().manual_seed(0)
    src = {"model.norm.weight": torch.randn(64, generator=g), "lm_head.weight": torch.randn(8, 64, generator=g),
           "a.trellis": torch.zeros(4, 4, dtype=torch.int16)}
    exp = {"model.norm.weight": src["model.norm.weight"].bfloat16(), "lm_head.weight": src["lm_head.weight"].bfloat16(),
           "a.trellis": src["a.trellis"]}
    d = tmp_path / "ckpt"
    d.mkdir()
    save_file(exp, str(d / "model-00001.safetensors"))
    return src, exp, d


def test_override_restores_source_precision(tmp_path, monkeypatch):
    src, exp, d = _export(tmp_path)
    path, sha = build_override(src, exp, ["model.norm.weight"], str(tmp_path), "org/model", "abc")
    merged, names = apply_override(hf_loader.open_dir(str(d)), path, sha)
    assert names == ["model.norm.weight"]
    assert merged["model.norm.weight"].dtype == torch.float32
    assert torch.equal(merged["model.norm.weight"], src["model.norm.weight"])
    assert merged["lm_head.weight"].dtype == torch.bfloat16 and len(merged) == 3
    # through the loader's environment switch
    from vllm_cmp170hx_b200 import envs

    monkeypatch.setenv("VLLM_EXL3_OVERRIDE", path)  # the reference's names are accepted
    monkeypatch.setenv("VLLM_EXL3_OVERRIDE_SHA256", sha)
    envs.reset_cache()
    try:
        t = hf_loader.open_dir(str(d), readahead=True)
        assert t["model.norm.weight"].dtype == torch.float32
    finally:
        monkeypatch.delenv("VLLM_EXL3_OVERRIDE")
        monkeypatch.delenv("VLLM_EXL3_OVERRIDE_SHA256")
        envs.reset_cache()


def test_override_refusals(tmp_path):
    src, exp, d = _export(tmp_path)
    tensors = hf_loader.open_dir(str(d))
    with pytest.raises(ValueError):  # not a cast of the source
        build_override({**src, "lm_head.weight": src["lm_head.weight"] + 1}, exp, ["lm_head.weight"], str(tmp_path))
    path, sha = build_override(src, exp, ["lm_head.weight"], str(tmp_path))
    with pytest.raises(ValueError):  # pin differs
        apply_override(tensors, path, "0" * 64)
    raw = json.loads(open(path).read())
    raw["tensors"][0]["sha256"] = "1" * 64
    bad = os.path.join(tmp_path, "bad.json")
    open(bad, "w").write(json.dumps(raw))
    import hashlib

    with pytest.raises(ValueError, match="do not hash to the manifest"):
        apply_override(tensors, bad, hashlib.sha256(open(bad, "rb").read()).hexdigest())
    raw = json.loads(open(path).read())
    raw["tensors"][0]["name"] = "a.trellis"
    open(bad, "w").write(json.dumps(raw))
    with pytest.raises(ValueError):  # packed part (and the sidecar lists another tensor)
        apply_override(tensors, bad, hashlib.sha256(open(bad, "rb").read()).hexdigest())


def test_readahead_runs(tmp_path):
    _, _, d = _export(tmp_path)
    with Readahead([str(p) for p in d.iterdir()]) as r:
        pass
    assert r.done.is_set()
