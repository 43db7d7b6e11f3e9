"""What a launch runs: the engine tree's state, the native extension's identity and the checkpoint's.

The reference's launcher checks the tree it launches (vllm_sm80/launch/treestate.py:312: tracked vs
unowned files, native-build provenance) and the checkpoint's completeness and identity against a
manifest with hash stamps (launch/checkpoint.py:213, schemas checkpoint-manifest/1 and
checkpoint-stamp/1), and writes both into the launch receipt.  The same three facts here, for this
package's single tree and in-tree extension:

* :func:`tree_state` -- the git commit of the package's tree and whether it is dirty (modified or
  untracked files outside the ignored build outputs); a tree without git reports no commit;
* :func:`native_identity` -- the built ``_C`` extension: its file, sha256, the ABI stamp it was built
  with, and whether any ``csrc`` source is newer than it (a stale build);
* :func:`checkpoint_manifest` / :func:`verify_checkpoint` -- a manifest of every file a checkpoint
  directory serves (``config.json``, the index and every weight shard it names, size and sha256), and a
  check against it: ``verified``, ``incomplete`` (a file missing, empty or of another size), ``mismatch``
  (a sha256 differs) or ``absent``.  Hashes are recorded once in a stamp beside the manifest (per file:
  device, inode, size, mtime_ns, ctime_ns, sha256); a later check re-hashes only files whose identity
  changed.  Exit codes of the command line: 0 verified, 4 incomplete, 5 mismatch, 6 absent.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
ROOT = PKG.parent

MANIFEST_SCHEMA = "checkpoint-manifest/1"
STAMP_SCHEMA = "checkpoint-stamp/1"
EXIT = {"verified": 0, "incomplete": 4, "mismatch": 5, "absent": 6}


def sha256_file(path: Path, chunk: int = 1 << 24) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(chunk)
            if not b:
                return h.hexdigest()
            h.update(b)


def _git(*args: str) -> str | None:
    try:
        r = subprocess.run(["git", "-C", str(ROOT), *args], capture_output=True, text=True, timeout=20)
    except (OSError, subprocess.TimeoutExpired):
        return None
    return r.stdout if r.returncode == 0 else None


def tree_state() -> dict:
    """{"commit", "dirty", "changed"}: the package tree's HEAD and the paths git reports as modified or
    untracked (ignored files -- build outputs, caches -- are not listed by git and do not count)."""
    head = _git("rev-parse", "HEAD")
    if head is None:
        return {"commit": None, "dirty": None, "changed": [], "reason": "not a git checkout"}
    status = _git("status", "--porcelain", "--untracked-files=all") or ""
    changed = [line[3:] for line in status.splitlines() if line.strip()]
    return {"commit": head.strip(), "dirty": bool(changed), "changed": changed[:200]}


def native_identity() -> dict:
    """The in-tree ``_C`` extension: path, sha256, ABI stamp, and whether a csrc source is newer."""
    libs = sorted(PKG.glob("_C*.so"))
    if not libs:
        return {"path": None, "reason": "no built extension (python setup.py build_ext --inplace)"}
    lib = libs[-1]
    from .. import _ext

    src = [p for p in (PKG / "csrc").iterdir() if p.suffix in (".cu", ".cuh", ".cpp", ".h")]
    newest = max((p.stat().st_mtime for p in src), default=0.0)
    return {"path": str(lib.relative_to(ROOT)), "sha256": sha256_file(lib), "build_info": _ext.EXPECTED_BUILD_INFO,
            "stale": newest > lib.stat().st_mtime,
            "newer_sources": sorted(p.name for p in src if p.stat().st_mtime > lib.stat().st_mtime)}


# ------------------------------------------------------------------------------------------ checkpoints
def checkpoint_files(path: Path) -> list[str]:
    """The files a checkpoint directory serves: config.json, the weight index and every shard it names,
    or the single weights file of an index-less checkpoint, plus any other *.safetensors / *.json."""
    names = set()
    for n in ("config.json", "tokenizer.json", "tokenizer_config.json", "generation_config.json"):
        if (path / n).exists():
            names.add(n)
    for idx in path.glob("*.index.json"):
        names.add(idx.name)
        names.update(json.loads(idx.read_text()).get("weight_map", {}).values())
    names.update(p.name for p in path.glob("*.safetensors"))
    return sorted(names)


def checkpoint_manifest(path: Path) -> dict:
    path = Path(path)
    files = {n: {"size": (path / n).stat().st_size, "sha256": sha256_file(path / n)} for n in checkpoint_files(path)}
    body = {"schema": MANIFEST_SCHEMA, "files": files}
    body["manifest_sha256"] = hashlib.sha256(json.dumps(files, sort_keys=True).encode()).hexdigest()
    return body


def _identity(st: os.stat_result) -> list[int]:
    return [st.st_dev, st.st_ino, st.st_size, st.st_mtime_ns, st.st_ctime_ns]


def verify_checkpoint(path: Path, manifest: dict, stamp_path: Path | None = None) -> tuple[str, dict]:
    """Check a checkpoint directory against its manifest.  Returns (status, {file: problem}); with a
    stamp path the per-file identities and hashes are read from and written to it, so files whose
    identity is unchanged are not hashed again."""
    path = Path(path)
    if manifest.get("schema") != MANIFEST_SCHEMA:
        raise ValueError(f"manifest schema {manifest.get('schema')!r}, expected {MANIFEST_SCHEMA}")
    if not path.is_dir():
        return "absent", {".": "no such directory"}
    stamp = {}
    if stamp_path is not None and Path(stamp_path).exists():
        s = json.loads(Path(stamp_path).read_text())
        if s.get("schema") == STAMP_SCHEMA and s.get("manifest_sha256") == manifest.get("manifest_sha256"):
            stamp = s.get("files", {})
    problems, hashed = {}, {}
    incomplete = False
    for name, want in manifest["files"].items():
        f = path / name
        if not f.exists() or (path / (name + ".incomplete")).exists():
            problems[name] = "missing"
            incomplete = True
            continue
        st = f.stat()
        if st.st_size == 0 or st.st_size != want["size"]:
            problems[name] = f"size {st.st_size}, manifest {want['size']}"
            incomplete = True
            continue
        ident = _identity(st)
        old = stamp.get(name)
        digest = old["sha256"] if old and old.get("identity") == ident else sha256_file(f)
        hashed[name] = {"identity": ident, "sha256": digest}
        if digest != want["sha256"]:
            problems[name] = "sha256 differs"
    status = "incomplete" if incomplete else ("mismatch" if problems else "verified")
    if stamp_path is not None and status == "verified":
        Path(stamp_path).write_text(json.dumps({"schema": STAMP_SCHEMA, "manifest_sha256":
                                                manifest["manifest_sha256"], "files": hashed}, indent=1))
    return status, problems


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="checkpoint manifests and checks; tree and native identity")
    sub = ap.add_subparsers(dest="cmd", required=True)
    m = sub.add_parser("manifest")
    m.add_argument("--path", required=True, type=Path)
    m.add_argument("--out", type=Path)
    v = sub.add_parser("verify")
    v.add_argument("--path", required=True, type=Path)
    v.add_argument("--manifest", required=True, type=Path)
    v.add_argument("--stamp", type=Path)
    sub.add_parser("tree")
    a = ap.parse_args(argv)
    if a.cmd == "manifest":
        text = json.dumps(checkpoint_manifest(a.path), indent=1)
        (a.out.write_text(text) if a.out else print(text))
        return 0
    if a.cmd == "verify":
        status, problems = verify_checkpoint(a.path, json.loads(a.manifest.read_text()), a.stamp)
        print(json.dumps({"status": status, "problems": problems}, indent=1))
        return EXIT[status]
    print(json.dumps({"tree": tree_state(), "native": native_identity()}, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
