"""Override sidecars and read-ahead for upstream-named checkpoints.

An exported (quantised) checkpoint may store some plain tensors at a lower precision than its
source (a norm weight cast fp32 -> bf16).  An override sidecar restores them: a safetensors file
with the source tensors plus a JSON manifest (format ``override-sidecar/2``, kept alike with the
reference's, vllm_sm80/kernels/exl3/override.py:1-13, so existing sidecars load)::

    {"format": "override-sidecar/2", "sidecar": "<file>.safetensors",
     "source": {"repo": ..., "revision": ...},
     "tensors": [{"name", "shape", "source_dtype", "export_dtype", "sha256",
                  "cast_check": {"export_dtype", "equal": true, "compared_elems"}}, ...]}

`apply_override` refuses, before replacing anything: a manifest whose sha256 differs from the
pinned one, a sidecar listing other tensors than the manifest, a tensor the checkpoint lacks or
holds at another dtype / shape, a packed EXL3 part, an entry without a passing cast check, a
sidecar tensor whose bytes do not hash to the recorded sha256, and a checkpoint tensor that is not
the sidecar tensor cast to the checkpoint's dtype bit for bit (only a precision difference, never
a changed value, is restored).  `build_override` writes a sidecar and manifest from the source
tensors.  `Readahead` asks the kernel to page a checkpoint's shards in ahead of the loader
(the reference's vllm_sm80/kernels/exl3/readahead.py).
"""

from __future__ import annotations

import hashlib
import json
import math
import os
import threading
from collections.abc import Mapping

import torch

FORMAT = "override-sidecar/2"
PACKED_SUFFIXES = (".trellis", ".suh", ".svh", ".mcg", ".mul1")
_DT = {torch.bool: "BOOL", torch.uint8: "U8", torch.int8: "I8", torch.int16: "I16", torch.float16: "F16",
       torch.bfloat16: "BF16", torch.int32: "I32", torch.float32: "F32", torch.int64: "I64", torch.float64: "F64"}
_TD = {v: k for k, v in _DT.items()}


def _bytes(t: torch.Tensor) -> bytes:
    return t.contiguous().view(torch.uint8).numpy().tobytes() if t.numel() else b""


def build_override(source: Mapping[str, torch.Tensor], export: Mapping[str, torch.Tensor], names: list[str],
                   out_dir: str, repo: str = "", revision: str = "", stem: str = "override") -> tuple[str, str]:
    """Write `stem`.safetensors with source[name] for `names` and its manifest; returns (manifest
    path, its sha256).  Every name must be a plain export tensor equal to the source cast to it."""
    from safetensors.torch import save_file

    entries, tensors = [], {}
    for n in names:
        s, e = source[n].contiguous(), export[n]
        if n.endswith(PACKED_SUFFIXES) or tuple(s.shape) != tuple(e.shape):
            raise ValueError(f"{n}: not a plain tensor of the export's shape")
        if not torch.equal(s.to(e.dtype).view(torch.uint8), e.contiguous().view(torch.uint8)):
            raise ValueError(f"{n}: the export is not the source cast to {e.dtype}")
        tensors[n] = s
        entries.append({"name": n, "shape": list(s.shape), "source_dtype": _DT[s.dtype], "export_dtype": _DT[e.dtype],
                        "sha256": hashlib.sha256(_bytes(s)).hexdigest(),
                        "cast_check": {"export_dtype": _DT[e.dtype], "equal": True, "compared_elems": s.numel()}})
    side = stem + ".safetensors"
    save_file(tensors, os.path.join(out_dir, side))
    raw = json.dumps({"format": FORMAT, "sidecar": side, "source": {"repo": repo, "revision": revision},
                      "tensors": entries}, indent=1).encode()
    path = os.path.join(out_dir, stem + ".json")
    with open(path, "wb") as f:
        f.write(raw)
    return path, hashlib.sha256(raw).hexdigest()


def apply_override(tensors: Mapping[str, torch.Tensor], manifest_path: str, sha256: str) -> tuple[Mapping, list[str]]:
    """The checkpoint's tensors with the sidecar's in place of the listed ones (all checks first)."""
    from safetensors import safe_open

    if not sha256:
        raise ValueError("apply_override: pass the expected sha256 of the manifest file (no digest was given)")
    with open(manifest_path, "rb") as f:
        raw = f.read()
    digest = hashlib.sha256(raw).hexdigest()
    if digest != sha256.lower():
        raise ValueError(f"{manifest_path}: file digest {digest} is not the expected {sha256.lower()}")
    spec = json.loads(raw)
    if spec.get("format") != FORMAT:
        raise ValueError(f"{manifest_path}: format {spec.get('format')!r} is not {FORMAT!r}")
    entries = spec["tensors"]
    names = [e["name"] for e in entries]
    side_path = os.path.join(os.path.dirname(manifest_path), spec["sidecar"])
    with safe_open(side_path, framework="pt") as h:
        side = {k: h.get_tensor(k) for k in h.keys()}
    if len(set(names)) != len(names) or set(names) != set(side):
        raise ValueError(f"{side_path}: its tensor names {sorted(side)} do not equal the manifest's {sorted(set(names))} (or a name repeats)")
    for e in entries:
        n, shape = e["name"], tuple(e["shape"])
        if n not in tensors:
            raise ValueError(f"{n}: listed for replacement but the checkpoint has no tensor of that name")
        if n.endswith(PACKED_SUFFIXES):
            raise ValueError(f"{n}: a packed EXL3 part (trellis / scales) cannot be replaced by a plain tensor")
        ex = tensors[n]
        if _DT[ex.dtype] != e["export_dtype"] or tuple(ex.shape) != shape:
            raise ValueError(f"{n}: the checkpoint holds {_DT[ex.dtype]} {tuple(ex.shape)}, the manifest expects {e['export_dtype']} {shape}")
        if e.get("cast_check") != {"export_dtype": e["export_dtype"], "equal": True, "compared_elems": math.prod(shape)}:
            raise ValueError(f"{n}: the manifest records no successful cast check over all {math.prod(shape)} elements")
        src = side[n]
        if _DT[src.dtype] != e["source_dtype"] or tuple(src.shape) != shape:
            raise ValueError(f"{n}: the sidecar holds {_DT[src.dtype]} {tuple(src.shape)}, the manifest lists {e['source_dtype']} {shape}")
        if hashlib.sha256(_bytes(src)).hexdigest() != e["sha256"]:
            raise ValueError(f"{n}: the sidecar bytes do not hash to the manifest's sha256")
        if not torch.equal(src.to(ex.dtype).view(torch.uint8), ex.contiguous().view(torch.uint8)):
            raise ValueError(f"{n}: casting the sidecar tensor to {ex.dtype} does not give the checkpoint's bytes")
    return _Overlay(tensors, {n: side[n] for n in names}), names


class _Overlay(Mapping):
    """`base` with some names replaced, still read lazily."""

    def __init__(self, base: Mapping, over: dict):
        self.base, self.over = base, over

    def __getitem__(self, k):
        return self.over[k] if k in self.over else self.base[k]

    def __contains__(self, k):
        return k in self.over or k in self.base

    def __iter__(self):
        return iter(self.base)

    def __len__(self):
        return len(self.base)


class Readahead:
    """Ask the kernel to read a checkpoint's shard files into the page cache on a background thread
    (POSIX_FADV_WILLNEED, file by file) while the loader starts on the first ones."""

    def __init__(self, paths: list[str]):
        self.paths = list(paths)
        self.done = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        try:
            for p in self.paths:
                fd = os.open(p, os.O_RDONLY)
                try:
                    os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_WILLNEED)
                finally:
                    os.close(fd)
        finally:
            self.done.set()

    def __enter__(self) -> "Readahead":
        self._t.start()
        return self

    def __exit__(self, *exc) -> None:
        self._t.join()
