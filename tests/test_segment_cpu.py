"""Table segment holder: files held in sealed memory by one process, attached by others (descriptor
passing over a Unix socket), leases, release modes, integrity checks, and the row reader reading a
held table through its descriptor."""

import hashlib
import os
import subprocess
import sys
import time

import pytest
import torch

from vllm_cmp170hx_b200.storage import segment, tables


def _write(path, data: bytes):
    with open(path, "wb") as f:
        f.write(data)
    return hashlib.sha256(data).hexdigest()


def _start(sock, label, files):
    args = [sys.executable, "-m", "vllm_cmp170hx_b200.storage.segment", "hold", "--socket", sock, "--label", label]
    for p, d in files:
        args += ["--file", f"{p}={d}"]
    proc = subprocess.Popen(args, cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    for _ in range(200):
        if os.path.exists(sock):
            break
        time.sleep(0.05)
    return proc


def _wait_ready(sock):
    for _ in range(200):
        st = segment.request(sock, {"op": "status"})
        if st["state"] != "filling":
            return st
        time.sleep(0.05)
    raise AssertionError("holder never got ready")


def test_hold_attach_map_and_drain(tmp_path):
    a = bytes(range(256)) * 9000
    b = os.urandom(3 << 20)
    pa, pb = str(tmp_path / "a.bin"), str(tmp_path / "b.bin")
    files = [(pa, _write(pa, a)), (pb, _write(pb, b))]
    sock = str(tmp_path / "h.sock")
    proc = _start(sock, "test", files)
    try:
        st = _wait_ready(sock)
        assert st["state"] == "ready" and st["clients"] == 0 and len(st["files"]) == 2
        att = segment.Attachment(sock, [pa, pb], timeout=10)
        m, off = att.map(pb, 123457, 1000)
        assert m[off:off + 1000] == b[123457:123457 + 1000]
        with open(att.fd_path(pa), "rb") as f:  # the descriptor reads like a file
            assert f.read() == a
        att2 = segment.Attachment(sock, [pa], timeout=10)
        assert segment.request(sock, {"op": "status"})["clients"] == 2
        # idle release refuses while attached; drain refuses new attaches and waits for the leases
        assert segment.request(sock, {"op": "release", "mode": "idle"})["exits"] is False
        assert segment.request(sock, {"op": "release", "mode": "drain"})["exits"] is False
        with pytest.raises(segment.SegmentError):
            segment.Attachment(sock, [pa], timeout=10)
        att2.close()
        assert proc.poll() is None
        m.close()
        att.close()
        assert proc.wait(timeout=20) == 0
    finally:
        if proc.poll() is None:
            proc.kill()


def test_bad_digest_exits_3(tmp_path):
    p = str(tmp_path / "x.bin")
    _write(p, b"abc" * 1000)
    sock = str(tmp_path / "bad.sock")
    proc = _start(sock, "bad", [(p, "0" * 64)])
    assert proc.wait(timeout=20) == segment.EXIT_BAD_FILE


def test_row_table_reads_a_held_file(tmp_path):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 256, generator=g)
    path = str(tmp_path / "rows.bin")
    tables.write_table(path, x)
    with open(path, "rb") as f:
        digest = hashlib.sha256(f.read()).hexdigest()
    sock = str(tmp_path / "rows.sock")
    proc = _start(sock, "rows", [(path, digest)])
    try:
        _wait_ready(sock)
        att = segment.Attachment(sock, [path], timeout=10)
        t = tables.RowTable(att.fd_path(path), 64, 256, cache_rows=16, threads=2)
        ids = torch.tensor([3, 63, 0])
        ref = tables.dequantize_rows(torch.from_numpy(tables.quantize_rows(x)), 256)[ids]
        assert torch.equal(t.lookup(ids).float(), ref.to(torch.bfloat16).float())
        att.close()
        assert segment.request(sock, {"op": "release", "mode": "force"})["exits"] is True
        assert proc.wait(timeout=20) == 0
    finally:
        if proc.poll() is None:
            proc.kill()


def test_manifest_hash_is_the_protocol_digest():
    """The digest is sha256 of the canonical JSON document {label, files: [{name, size, sha256}]}
    (sorted keys, no whitespace): clients of either holder compute the same value."""
    import hashlib

    from vllm_cmp170hx_b200.storage.segment import manifest_hash

    files = [{"name": "a.bin", "size": 3, "sha256": "ab" * 32}, {"name": "b.bin", "size": 0, "sha256": "cd" * 32}]
    text = ('{"files":[{"name":"a.bin","sha256":"' + "ab" * 32 + '","size":3},{"name":"b.bin","sha256":"'
            + "cd" * 32 + '","size":0}],"label":"L"}')
    assert manifest_hash("L", files) == hashlib.sha256(text.encode()).hexdigest()
