"""Sharded checkpoints of a built model: save every rank's tensors, reload them without re-drawing.

Layout of a checkpoint directory::

    manifest.json                       model config, parallel layout, per-rank tensor inventory
    model-rank{r}-of-{world}.safetensors  rank r's tensors, by module path

The tensors are stored exactly as the kernels consume them (EXL3 trellis
``int16 [K/16, N/16, 8*bits_x2]`` per expert with ``suh`` / ``svh``; Marlin
``int32 [E, K/16, 2N]`` with permuted ``bf16 [E, K/128, N]`` scales; fp8 weights
with 128x128 block scales; bf16 elsewhere), already cut for the rank's
tensor / pipeline / expert split, so loading is a straight copy.  ``load``
checks the manifest before touching the model: the same architecture, the
same parallel layout and, tensor by tensor, the same shapes and dtypes (the
reference's EXL3 manifest validates trellis geometry and accounts for every
tensor the same way, vllm_sm80/kernels/exl3/utils.py:183-290).
"""

from __future__ import annotations

import dataclasses
import json
import os

import torch

from .parallel import state as pstate

MANIFEST = "manifest.json"


def _containers(model: torch.nn.Module):
    """(path, dataclass instance) of the tensor containers that are not nn.Modules (experts, fp8 linears)."""
    for name, mod in model.named_modules():
        for attr in ("experts", "lin"):
            obj = getattr(mod, attr, None)
            if obj is not None and dataclasses.is_dataclass(obj) and not isinstance(obj, torch.nn.Module):
                yield (f"{name}.{attr}" if name else attr), obj


def collect(model: torch.nn.Module) -> dict[str, torch.Tensor]:
    out = {k: v for k, v in model.state_dict().items()}
    for path, obj in _containers(model):
        for f in dataclasses.fields(obj):
            v = getattr(obj, f.name)
            if isinstance(v, torch.Tensor):
                out[f"{path}.{f.name}"] = v
    return out


def _layout(st) -> dict:
    return {"world": st.world_size, "tp": st.tp_size, "pp": st.pp_size, "expert_parallel": bool(st.expert_parallel)}


def shard_file(rank: int, world: int) -> str:
    return f"model-rank{rank}-of-{world}.safetensors"


def save(model: torch.nn.Module, out_dir: str) -> str:
    """Write this rank's tensors; rank 0 also writes the manifest (every rank's inventory is gathered
    through the world CPU group when there is more than one rank)."""
    from safetensors.torch import save_file

    st = pstate.get()
    os.makedirs(out_dir, exist_ok=True)
    tensors = {k: v.detach().contiguous().cpu() for k, v in collect(model).items()}
    path = os.path.join(out_dir, shard_file(st.rank, st.world_size))
    save_file(tensors, path)
    inv = {k: {"shape": list(v.shape), "dtype": str(v.dtype).replace("torch.", "")} for k, v in tensors.items()}
    invs = [inv]
    if st.world_size > 1:
        import torch.distributed as dist

        invs = [None] * st.world_size
        dist.all_gather_object(invs, inv, group=st.world_cpu_group)
    if st.rank == 0:
        manifest = {"format": "vllm_cmp170hx_b200/sharded-1", "model": dataclasses.asdict(model.cfg),
                    "layout": _layout(st), "ranks": {str(r): i for r, i in enumerate(invs)}}
        with open(os.path.join(out_dir, MANIFEST), "w") as f:
            json.dump(manifest, f)
    return path


class CheckpointMismatch(ValueError):
    pass


def load(model: torch.nn.Module, in_dir: str, strict: bool = True) -> None:
    """Copy this rank's tensors into an already built model of the same architecture and layout."""
    from safetensors.torch import load_file

    st = pstate.get()
    with open(os.path.join(in_dir, MANIFEST)) as f:
        manifest = json.load(f)
    if manifest.get("layout") != _layout(st):
        raise CheckpointMismatch(f"parallel layout {manifest.get('layout')} != this run's {_layout(st)}")
    if manifest.get("model") != dataclasses.asdict(model.cfg):
        raise CheckpointMismatch("model configuration differs from the checkpoint's")
    saved = load_file(os.path.join(in_dir, shard_file(st.rank, st.world_size)))
    want = collect(model)
    missing = sorted(set(want) - set(saved))
    extra = sorted(set(saved) - set(want))
    if strict and (missing or extra):
        raise CheckpointMismatch(f"missing {missing[:5]}, unexpected {extra[:5]}")
    for name, dst in want.items():
        src = saved.get(name)
        if src is None:
            continue
        if tuple(src.shape) != tuple(dst.shape) or src.dtype != dst.dtype:
            raise CheckpointMismatch(f"{name}: saved {tuple(src.shape)} {src.dtype}, model {tuple(dst.shape)} "
                                     f"{dst.dtype}")
        with torch.no_grad():
            dst.copy_(src.to(dst.device))
    drop_decoded_caches(model)


def drop_decoded_caches(model: torch.nn.Module) -> None:
    """Forget the decoded-weight caches of the CPU reference path (stale once weights change)."""
    for _, obj in _containers(model):
        for attr in ("_dense_cache", "_dense"):
            if attr in vars(obj):
                object.__delattr__(obj, attr)
