"""Storage-backed row tables on the host: native threaded reader + set-associative LRU cache,
retries and failed-row poisoning (faults injected on the host, never on a device)."""

import numpy as np
import torch

from vllm_cmp170hx_b200 import _ext
from vllm_cmp170hx_b200.storage import tables


def _table(tmp_path, n=300, dim=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, dim, generator=g) * 3
    path = str(tmp_path / "t.bin")
    tables.write_table(path, x)
    return path, x


def test_rows_roundtrip_and_cache(tmp_path):
    path, x = _table(tmp_path)
    t = tables.RowTable(path, 300, 256, cache_rows=64, ways=4, threads=4)
    ids = torch.tensor([5, 17, 299, 5, 0, 128])
    y = t.lookup(ids).float()
    ref = tables.dequantize_rows(torch.from_numpy(tables.quantize_rows(x)), 256)[ids]
    assert torch.equal(y, ref.to(torch.bfloat16).float())
    assert ((y - x[ids]).abs() / x[ids].abs().clamp_min(1e-3)).median() < 0.08  # e4m3 precision
    hits0, misses0 = t.cache.stats()
    t.lookup(ids)
    hits1, misses1 = t.cache.stats()
    assert misses1 == misses0 and hits1 - hits0 == 6
    # eviction: more distinct rows than the cache holds, all still correct
    big = torch.arange(0, 300, 2)
    full = tables.dequantize_rows(torch.from_numpy(tables.quantize_rows(x)), 256)
    assert torch.equal(t.lookup(big).float(), full[big].to(torch.bfloat16).float())


def test_failed_rows_are_poisoned_and_retried(tmp_path):
    path, x = _table(tmp_path, seed=1)
    t = tables.RowTable(path, 300, 256, cache_rows=64, threads=2, retries=2)
    t.reader.fail_rows_for_test([7, 8])
    y = t.lookup(torch.tensor([6, 7, 8, 9])).float()
    assert torch.isnan(y[1]).all() and torch.isnan(y[2]).all() and torch.isfinite(y[[0, 3]]).all()
    reads, retries, failures, _ = t.reader.stats()
    assert failures == 2 and retries == 4  # 2 retries for each failed row
    t.reader.fail_rows_for_test([])  # the failed rows were not cached: a later step reads them again
    assert torch.isfinite(t.lookup(torch.tensor([7, 8])).float()).all()
    bad = t.lookup(torch.tensor([1000]))  # out of range is a failed row, not a crash
    assert torch.isnan(bad.float()).all()
