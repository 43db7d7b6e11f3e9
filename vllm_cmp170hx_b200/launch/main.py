"""Resolve layered launch settings into one validated server command.

    python -m vllm_cmp170hx_b200.launch.main --settings DIR --layout tp4 \
        [--overlay NAME ...] [--set engine.max-num-seqs=128 ...] [--dry-run]

Layers, lowest first (the reference's resolver order, vllm_sm80/launch/
resolver.py:433: defaults -> model -> layout -> variants/overlays -> --set):
  1. ``launch/defaults.toml`` of this package;
  2. ``DIR/model.toml``  (``model = "config3" | checkpoint dir``, tokenizer, engine knobs);
  3. ``DIR/layouts/<layout>.toml`` (tp, engine sizes);
  4. ``DIR/overlays/<name>.toml`` for each ``--overlay``;
  5. ``--set section.key=value`` (value parsed as TOML).
Every ``[env]`` name must be declared in vllm_cmp170hx_b200.envs (or be a
reference alias); retired sm_80 switches are refused.  The result is
printed as JSON (``--dry-run``) or exec'ed: ``torchrun`` when tp > 1.
A receipt (resolved settings + sha256 of every input file, the engine tree's
commit and dirty state, the native extension's identity and the checkpoint's
manifest digest) is written beside the command when ``--receipt PATH`` is
given.  ``--require-clean`` refuses a dirty tree or a native build older than
its sources; ``--checkpoint-manifest FILE`` refuses a checkpoint directory
that is not complete and identical to the manifest (launch/provenance.py).
"""

from __future__ import annotations

import argparse
import copy
import hashlib
import json
import os
import sys
import tomllib
from pathlib import Path

from .. import envs

HERE = Path(__file__).parent


class LaunchError(ValueError):
    pass


def _merge(a: dict, b: dict) -> dict:
    out = copy.deepcopy(a)
    for k, v in b.items():
        if isinstance(v, dict) and isinstance(out.get(k), dict):
            out[k] = _merge(out[k], v)
        else:
            out[k] = v
    return out


def _load(path: Path) -> dict:
    try:
        return tomllib.loads(path.read_text())
    except FileNotFoundError:
        raise LaunchError(f"missing settings file {path}") from None


def resolve(settings: Path, layout: str, overlays: list[str] = (), sets: list[str] = ()) -> tuple[dict, list[Path]]:
    files = [HERE / "defaults.toml", settings / "model.toml", settings / "layouts" / f"{layout}.toml"]
    files += [settings / "overlays" / f"{o}.toml" for o in overlays]
    cfg: dict = {}
    for f in files:
        cfg = _merge(cfg, _load(f))
    for s in sets:
        if "=" not in s or "." not in s.split("=", 1)[0]:
            raise LaunchError(f"--set wants section.key=value, got {s!r}")
        path, val = s.split("=", 1)
        sec, key = path.split(".", 1)
        try:
            v = tomllib.loads(f"v = {val}")["v"]
        except tomllib.TOMLDecodeError:
            v = val
        cfg.setdefault(sec, {})[key] = v
    if "model" not in cfg:
        raise LaunchError("model.toml must name `model`")
    for name in cfg.get("env", {}):
        if any(name.startswith(p) for p in envs.RETIRED_PREFIXES):
            raise LaunchError(f"{name} switches an sm_80-only path of the reference; remove it")
        if name.startswith("VLLM_") and name not in envs.VARS and name not in envs.ALIASES:
            raise LaunchError(f"unknown variable {name}")
    return cfg, files


def command(cfg: dict) -> tuple[list[str], dict[str, str]]:
    tp = int(cfg.get("launch", {}).get("tp", 1))
    server = [sys.executable, "-m", "vllm_cmp170hx_b200.api.server", "--model", str(cfg["model"]), "--tp", str(tp)]
    if cfg.get("tokenizer"):
        server += ["--tokenizer", str(cfg["tokenizer"])]
    for k, v in sorted(cfg.get("engine", {}).items()):
        if isinstance(v, bool):
            if v:
                server.append(f"--{k}")
        else:
            server += [f"--{k}", str(v)]
    if tp > 1:
        port = str(cfg.get("launch", {}).get("master-port", 29512))
        argv = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
                "--master-addr", "127.0.0.1", "--master-port", port] + server[1:]
    else:
        argv = server
    env = {k: str(v) for k, v in cfg.get("env", {}).items()}
    return argv, env


def receipt(cfg: dict, files: list[Path], argv: list[str], env: dict, checkpoint: dict | None = None) -> dict:
    from . import provenance

    return {"settings": cfg, "argv": argv, "env": env,
            "inputs": {str(f): hashlib.sha256(f.read_bytes()).hexdigest() for f in files if f.exists()},
            "tree": provenance.tree_state(), "native": provenance.native_identity(), "checkpoint": checkpoint}


def check_launch(cfg: dict, require_clean: bool, manifest_path: Path | None) -> dict | None:
    """Provenance gates before the exec: with `require_clean` a dirty tree or a stale native build is
    refused; with a manifest the model directory must verify against it (its stamp is kept beside the
    manifest).  Returns the checkpoint record for the receipt."""
    from . import provenance

    if require_clean:
        t = provenance.tree_state()
        if t["dirty"]:
            raise LaunchError(f"the engine tree is dirty ({len(t['changed'])} changed files, e.g. {t['changed'][:3]})")
        n = provenance.native_identity()
        if n.get("path") is None or n.get("stale"):
            raise LaunchError(f"the native extension is missing or older than its sources: {n}")
    if manifest_path is None:
        return None
    manifest = json.loads(Path(manifest_path).read_text())
    stamp = Path(str(manifest_path) + ".stamp.json")
    status, problems = provenance.verify_checkpoint(Path(str(cfg["model"])), manifest, stamp)
    if status != "verified":
        raise LaunchError(f"checkpoint {cfg['model']} is {status}: {problems}")
    return {"path": str(cfg["model"]), "manifest_sha256": manifest["manifest_sha256"], "status": status}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--settings", required=True, type=Path)
    ap.add_argument("--layout", required=True)
    ap.add_argument("--overlay", action="append", default=[])
    ap.add_argument("--set", action="append", default=[])
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--receipt", type=Path)
    ap.add_argument("--require-clean", action="store_true", help="refuse a dirty tree or a stale native build")
    ap.add_argument("--checkpoint-manifest", type=Path, help="verify the model directory against this manifest")
    a = ap.parse_args(argv)
    cfg, files = resolve(a.settings, a.layout, a.overlay, a.set)
    cmd, env = command(cfg)
    ck = check_launch(cfg, a.require_clean, a.checkpoint_manifest)
    rec = receipt(cfg, files, cmd, env, ck)
    if a.receipt:
        a.receipt.write_text(json.dumps(rec, indent=2, default=str))
    if a.dry_run:
        print(json.dumps({"argv": cmd, "env": env}, indent=2))
        return
    os.execvpe(cmd[0], cmd, {**os.environ, **env})


if __name__ == "__main__":
    main()
