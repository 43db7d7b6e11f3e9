"""Size cut-offs of the kernels, read from a per-card table.

A speed crossover (a split count, a tile size, the largest message a
transport takes) is data, not code: ``tuning/<card>.toml`` holds rows of
(op, param, key, value, evidence) and the code asks :func:`lookup` for the
value at its own shape -- the same contract as the reference's
vllm_sm80/tuning.py:222 (most-specific key wins, equally specific matches
are a table error, cached per query, a miss logs once and returns the
default).  The table is ``VLLM_B200_TUNING_FILE`` when set, else the file
named after the current device (lower-case, non-alphanumerics -> '-').

    schema = "b200-tuning/1"
    card = "NVIDIA B200"
    [[row]]
    op = "gemm_bf16"; param = "splitk"; key = {n = 2304, k = 4096}; value = 8
    evidence = "where the number comes from"
"""

from __future__ import annotations

import functools
import logging
import re
import tomllib
from dataclasses import dataclass
from pathlib import Path

from . import envs

log = logging.getLogger(__name__)
SCHEMA = "b200-tuning/1"
TABLE_DIR = Path(__file__).with_name("tuning")


class TuningTableError(ValueError):
    pass


@dataclass(frozen=True)
class Row:
    op: str
    param: str
    key: tuple
    value: int | float | str
    evidence: str


def card_file(device_name: str) -> Path:
    return TABLE_DIR / (re.sub(r"[^a-z0-9]+", "-", device_name.lower()).strip("-") + ".toml")


def _frozen(v):
    """Array values as (nested) tuples: rows are hashable and their values immutable."""
    return tuple(_frozen(x) for x in v) if isinstance(v, list) else v


def parse(text: str, source: str = "<table>") -> list[Row]:
    d = tomllib.loads(text)
    if d.get("schema") != SCHEMA:
        raise TuningTableError(f"{source}: schema must be {SCHEMA!r}")
    extra = set(d) - {"schema", "card", "row"}
    if extra:
        raise TuningTableError(f"{source}: unknown top-level fields {sorted(extra)}")
    rows = []
    for i, r in enumerate(d.get("row", [])):
        if set(r) != {"op", "param", "key", "value", "evidence"}:
            raise TuningTableError(f"{source}: row {i} must have exactly op, param, key, value, evidence")
        rows.append(Row(r["op"], r["param"], tuple(sorted(r["key"].items())), _frozen(r["value"]), r["evidence"]))
    return rows


@functools.cache
def _table() -> tuple[Row, ...]:
    path = envs.get("VLLM_B200_TUNING_FILE")
    if not path:
        try:
            import torch

            if not torch.cuda.is_available():
                return ()
            path = str(card_file(torch.cuda.get_device_name()))
        except Exception:  # noqa: BLE001
            return ()
    p = Path(path)
    if not p.exists():
        return ()
    return tuple(parse(p.read_text(), str(p)))


def lookup(op: str, param: str, key: dict, default, rows: tuple[Row, ...] | None = None):
    rows = _table() if rows is None else rows
    return _lookup(rows, op, param, tuple(sorted(key.items())), default)


@functools.cache
def _lookup(rows, op, param, key, default):
    kd = dict(key)
    best, best_n, tie = None, -1, False
    for r in rows:
        if r.op != op or r.param != param:
            continue
        if all(kd.get(k) == v for k, v in r.key):
            n = len(r.key)
            if n > best_n:
                best, best_n, tie = r, n, False
            elif n == best_n:
                tie = True
    if tie:
        raise TuningTableError(f"two rows of equal specificity match {op}/{param} at {kd}")
    if best is None:
        log.info("tuning: no row for %s/%s at %s; using %r", op, param, kd, default)
        return default
    return best.value
