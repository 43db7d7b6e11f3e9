"""EXL3-coded PLE tables on the host: the oracle against a bit-by-bit restatement of the format,
the table file round trip through the native row reader (owner ranges, head gaps, failed reads)
and the tensor-parallel sum over two gloo ranks (reference: models/qwen4_exp/exl3_ple.py)."""

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from vllm_cmp170hx_b200.formats import ple as fple


def _scalar_value(trellis_row, c, dim, bits, scale, bias):
    state = 0
    for m in range(16):
        src = (c - m // bits) % dim
        rb = src * bits + m % bits
        word = int(trellis_row[1 + rb // 16]) & 0xFFFF
        state |= ((word >> (rb % 16)) & 1) << m
    p = (state * 0x83DCD12D) & 0xFFFFFFFF
    s = sum((p >> (8 * i)) & 255 for i in range(4))
    a = np.array([0x1EEE], np.uint16).view(np.float16)[0]
    b = np.array([0xC931], np.uint16).view(np.float16)[0]
    v = np.float16(np.float32(1024 + s) * np.float32(a) + np.float32(b))
    y = np.float32(np.float32(v) * np.float32(scale)) + np.float32(bias)
    return torch.tensor(float(np.float32(y))).to(torch.bfloat16).item()


@pytest.mark.parametrize("dim,bits", [(16, 1), (32, 3), (64, 4), (48, 8), (16, 16), (80, 5)])
def test_oracle_matches_bitwise_restatement(dim, bits):
    t = fple.random_table(heads=2, vocab=5, dim=dim, bits=bits, seed=dim + bits)
    ids = torch.tensor([0, 3, 7, 9])
    y = fple.decode_rows(t["trellis"][ids], ids, t["head_bias"], t["head_offsets"], t["head_vocab_sizes"], 0, 10, bits)
    for i, r in enumerate(ids.tolist()):
        h = r // 5
        scale = t["trellis"][r, 0].view(torch.float16).item()
        for c in range(0, dim, 7):
            exp = _scalar_value(t["trellis"][r], c, dim, bits, scale, t["head_bias"][h, c].item())
            assert y[i, c].item() == exp, (r, c)


def test_oracle_masks_owner_range_gaps_and_failed_rows():
    t = fple.random_table(heads=2, vocab=6, dim=32, bits=4, padding=4)
    ids = torch.tensor([1, 7, 12, 13, 2])  # 12, 13 are padding rows after the last head
    failed = torch.tensor([0, 0, 0, 0, 1], dtype=torch.uint8)
    y = fple.decode_rows(t["trellis"][ids], ids, t["head_bias"], t["head_offsets"], t["head_vocab_sizes"], 0, 6, 4,
                         failed)
    assert y[0].abs().sum() > 0
    assert (y[1] == 0).all()  # owned by another rank
    assert (y[2] == 0).all() and (y[3] == 0).all()  # no head holds them
    assert y[4].isnan().all()


def _write(tmp_path, **kw):
    t = fple.random_table(**kw)
    path = os.path.join(tmp_path, "ngram_embedding.safetensors")
    fple.write_table(path, "model.ngram_embedding", t, kw["bits"])
    return path, t


def test_layout_and_table_lookup_round_trip(tmp_path):
    from vllm_cmp170hx_b200.storage.ple import PleTable

    path, t = _write(tmp_path, heads=3, vocab=40, dim=64, bits=4, padding=8)
    lay = fple.read_layout(path, "model.ngram_embedding")
    assert (lay.rows, lay.dim, lay.heads, lay.bits, lay.words) == (128, 64, 3, 4, 17)
    raw = np.fromfile(path, dtype=np.uint8)[lay.base:lay.base + lay.rows * lay.row_bytes]
    assert torch.equal(torch.from_numpy(raw.copy()).view(torch.int16).view(lay.rows, lay.words), t["trellis"])

    tab = PleTable(path, "model.ngram_embedding", cache_rows=64, ways=4, threads=2)
    ids = torch.tensor([[0, 40, 80], [39, 79, 119], [5, 45, 85], [0, 40, 80]])
    rows, failed = tab.lookup(ids)
    assert rows.shape == (4, 3 * 64) and not failed.any()
    flat = ids.reshape(-1)
    exp = fple.decode_rows(t["trellis"][flat], flat, t["head_bias"], t["head_offsets"], t["head_vocab_sizes"], 0, 128,
                           4).view(4, -1)
    assert torch.equal(rows, exp)
    rows2, _ = tab.lookup(ids)  # a second lookup is served from the host cache
    assert torch.equal(rows2, exp) and tab.stats()["hits"] >= 12

    # a read that fails after its retries poisons its token, which comes back zeroed and flagged
    tab.reader.fail_rows_for_test([46])  # a row not in the host cache yet
    ids[2, 1] = 46
    rows, failed = tab.lookup(ids)
    assert failed.tolist() == [False, False, True, False]
    assert (rows[2] == 0).all() and torch.equal(rows[0], exp[0])


def _tp_worker(rank, world, path, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from vllm_cmp170hx_b200.storage.ple import PleTable

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        lay = fple.read_layout(path, "p")
        per = (lay.rows + world - 1) // world
        tab = PleTable(path, "p", rank * per, min(lay.rows, (rank + 1) * per), threads=2, group=dist.group.WORLD)
        if rank == 1:
            tab.reader.fail_rows_for_test([70])
        ids = torch.tensor([[3, 50], [63, 64], [10, 70]])
        rows, failed = tab.lookup(ids)
        q.put((rank, rows, failed))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_sum_over_owner_ranges(tmp_path):
    t = fple.random_table(heads=2, vocab=64, dim=32, bits=2)
    path = os.path.join(tmp_path, "t.safetensors")
    fple.write_table(path, "p", t, 2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, path, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    flat = torch.tensor([3, 50, 63, 64, 10, 70])
    exp = fple.decode_rows(t["trellis"][flat], flat, t["head_bias"], t["head_offsets"], t["head_vocab_sizes"], 0, 128,
                           2).view(3, -1)
    for rank, rows, failed in res:
        # row 70 is rank 1's and its read failed: every rank flags token 2
        assert failed.tolist() == [False, False, True], rank
        assert torch.equal(rows[:2], exp[:2]) and (rows[2] == 0).all(), rank
