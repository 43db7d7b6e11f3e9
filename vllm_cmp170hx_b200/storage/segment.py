"""Read-only host images of large table files, held by one process across server restarts.

A holder process reads each named file once into a sealed memory file (``memfd``) and hands
read-only descriptors to the servers that attach, so a restarted server maps the bytes instead of
reading tens of GiB from storage again.  Standard library only; runs as a script:

    python -m vllm_cmp170hx_b200.storage.segment hold --socket SOCK --label L --file PATH=SHA256 [...]
    python -m vllm_cmp170hx_b200.storage.segment status --socket SOCK
    python -m vllm_cmp170hx_b200.storage.segment release --socket SOCK [--mode idle|drain|force]

Protocol (kept alike with the reference's holder, vllm_sm80/table_segment.py:1-45, so existing
launch scripts and clients work): ``AF_UNIX`` ``SOCK_SEQPACKET``, one JSON object per message.
``status`` reports the state (``filling`` / ``ready`` / ``draining``), the held files with their
identity and digest, the manifest hash and the attached clients; ``release`` with mode ``idle``
(exit when nobody is attached), ``drain`` (refuse new attaches, exit when the last client leaves)
or ``force`` (exit now; existing mappings stay valid); ``attach`` with the identities the client
expects, answered once the fill is done with the descriptors (``SCM_RIGHTS``); the connection is
the client's lease.

The fill checks the file's sha256 and that the file did not change while it was read (device,
inode, size, modification time), then seals the memory file against writes and resizes.  A file
that fails the checks makes ``hold`` exit with status 3.

``Attachment(socket, paths).map(path, offset, nbytes)`` returns a read-only mapping of a byte range;
``Attachment.fd_path(path)`` names the descriptor as a file for readers that take a path (the native
row reader of ``storage/tables.py`` preads it like any file).
"""

from __future__ import annotations

import argparse
import array
import fcntl
import hashlib
import json
import mmap
import os
import selectors
import signal
import socket
import sys
import threading
from dataclasses import dataclass, field

VERSION = 1
MAX_MESSAGE = 64 << 10
CHUNK = 16 << 20
F_ADD_SEALS = getattr(fcntl, "F_ADD_SEALS", 1033)
F_GET_SEALS = getattr(fcntl, "F_GET_SEALS", 1034)
SEALS = (getattr(fcntl, "F_SEAL_SEAL", 0x1) | getattr(fcntl, "F_SEAL_SHRINK", 0x2)
         | getattr(fcntl, "F_SEAL_GROW", 0x4) | getattr(fcntl, "F_SEAL_WRITE", 0x8))
EXIT_BAD_FILE = 3


class SegmentError(RuntimeError):
    pass


def file_identity(path: str) -> dict:
    """What a client and the holder agree a file is: its resolved path, device, inode, size and
    modification time (the identity fields of the protocol)."""
    real = os.path.realpath(path)
    st = os.stat(real)
    return {"path": real, "dev": st.st_dev, "ino": st.st_ino, "size": st.st_size, "mtime_ns": st.st_mtime_ns}


def manifest_hash(label: str, files: list[dict]) -> str:
    """The manifest digest of the protocol: sha256 over the canonical JSON text (keys sorted, no
    whitespace) of ``{"label": label, "files": [{"name", "size", "sha256"}, ...]}`` with the files in
    holding order, so a client of either holder computes the same value."""
    listed = [{k: f[k] for k in ("name", "size", "sha256")} for f in files]
    canonical = json.dumps({"files": listed, "label": label}, sort_keys=True, separators=(",", ":"))
    return hashlib.sha256(canonical.encode()).hexdigest()


def _send(sock: socket.socket, obj: dict, fds: list[int] | None = None) -> None:
    data = json.dumps(obj).encode()
    if len(data) > MAX_MESSAGE:
        raise SegmentError("message too large")
    if fds:
        sock.sendmsg([data], [(socket.SOL_SOCKET, socket.SCM_RIGHTS, array.array("i", fds))])
    else:
        sock.send(data)


def _recv(sock: socket.socket, maxfds: int = 0) -> tuple[dict, list[int]]:
    fds = array.array("i")
    data, anc, _, _ = sock.recvmsg(MAX_MESSAGE, socket.CMSG_LEN(maxfds * fds.itemsize) if maxfds else 0)
    for level, typ, payload in anc:
        if level == socket.SOL_SOCKET and typ == socket.SCM_RIGHTS:
            fds.frombytes(payload[:len(payload) - len(payload) % fds.itemsize])
    if not data:
        raise SegmentError("holder closed the connection")
    return json.loads(data.decode()), list(fds)


def _connect(path: str, timeout: float | None) -> socket.socket:
    s = socket.socket(socket.AF_UNIX, socket.SOCK_SEQPACKET)
    s.settimeout(timeout)
    s.connect(path)
    return s


def request(path: str, obj: dict, timeout: float | None = 10.0) -> dict:
    """One request / answer exchange with a holder."""
    with _connect(path, timeout) as s:
        _send(s, obj)
        return _recv(s)[0]


@dataclass
class HeldFile:
    path: str
    sha256: str
    identity: dict = field(default_factory=dict)
    fd: int = -1
    filled: int = 0


class Holder:
    """Fills the memory files, then serves status / release / attach on the socket."""

    def __init__(self, socket_path: str, label: str, files: list[tuple[str, str]]):
        self.socket_path, self.label = socket_path, label
        self.files = [HeldFile(p, d.lower()) for p, d in files]
        self.state = "filling"
        self.error: str | None = None
        self.clients: dict[int, socket.socket] = {}
        self.pending: list[tuple[socket.socket, dict]] = []
        self.exit_when_idle = False
        self._lock = threading.Lock()
        self._done = threading.Event()

    # ------------------------------------------------------------------ fill
    def _fill_one(self, hf: HeldFile) -> None:
        before = file_identity(hf.path)
        hf.identity = before
        size = before["size"]
        fd = os.memfd_create("table:" + os.path.basename(before["path"]), os.MFD_CLOEXEC | getattr(os, "MFD_ALLOW_SEALING", 2))
        os.ftruncate(fd, size)
        h = hashlib.sha256()
        with open(hf.path, "rb", buffering=0) as src:
            off = 0
            while off < size:
                buf = src.read(min(CHUNK, size - off))
                if not buf:
                    raise SegmentError(f"{hf.path}: short read at {off}")
                h.update(buf)
                os.pwrite(fd, buf, off)
                off += len(buf)
                with self._lock:
                    hf.filled = off
        after = file_identity(hf.path)
        if after != before:
            raise SegmentError(f"{hf.path} changed while it was read")
        if h.hexdigest() != hf.sha256:
            raise SegmentError(f"{hf.path}: sha256 {h.hexdigest()} != {hf.sha256}")
        fcntl.fcntl(fd, F_ADD_SEALS, SEALS)
        hf.fd = fd

    def fill(self) -> None:
        try:
            for hf in self.files:
                self._fill_one(hf)
            with self._lock:
                self.state = "ready"
        except (OSError, SegmentError) as e:
            with self._lock:
                self.error = str(e)
                self.state = "failed"
        finally:
            self._done.set()

    # ------------------------------------------------------------------ answers
    def manifest(self) -> str:
        return manifest_hash(self.label, [{"name": os.path.basename(f.path),
                                           "size": f.identity.get("size", 0), "sha256": f.sha256}
                                          for f in self.files])

    def status(self) -> dict:
        with self._lock:
            return {"version": VERSION, "state": self.state, "label": self.label, "error": self.error,
                    "manifest": self.manifest(), "clients": len(self.clients),
                    "files": [{"path": f.path, "identity": f.identity, "sha256": f.sha256,
                               "filled": f.filled} for f in self.files]}

    def _attach_answer(self, msg: dict) -> tuple[dict, list[int]]:
        want = msg.get("files", [])
        by_path = {f.identity["path"]: f for f in self.files}
        fds, names = [], []
        for ident in want:
            f = by_path.get(ident.get("path"))
            if f is None or {k: ident.get(k) for k in f.identity} != f.identity:
                return {"ok": False, "error": f"not held (or changed): {ident.get('path')}"}, []
            fds.append(f.fd)
            names.append(f.identity["path"])
        return {"ok": True, "files": names, "manifest": self.manifest()}, fds

    # ------------------------------------------------------------------ serve
    def serve(self) -> int:
        try:
            os.unlink(self.socket_path)
        except FileNotFoundError:
            pass
        srv = socket.socket(socket.AF_UNIX, socket.SOCK_SEQPACKET)
        srv.bind(self.socket_path)
        srv.listen(64)
        srv.setblocking(False)
        filler = threading.Thread(target=self.fill, daemon=True)
        filler.start()
        sel = selectors.DefaultSelector()
        sel.register(srv, selectors.EVENT_READ, None)
        stop = {"now": False}
        signal.signal(signal.SIGTERM, lambda *_: stop.update(now=True))
        rc = 0
        try:
            while not stop["now"]:
                for key, _ in sel.select(timeout=0.05):
                    if key.data is None:
                        conn, _ = srv.accept()
                        sel.register(conn, selectors.EVENT_READ, "client")
                    else:
                        if self._handle(sel, key.fileobj, stop):
                            break
                if self._done.is_set():
                    if self.state == "failed":
                        for conn, _ in self.pending:
                            _send(conn, {"ok": False, "error": self.error})
                        rc = EXIT_BAD_FILE
                        break
                    for conn, msg in self.pending:
                        answer, fds = self._attach_answer(msg)
                        _send(conn, answer, fds)
                        if answer["ok"]:
                            self.clients[conn.fileno()] = conn
                    self.pending.clear()
                if self.exit_when_idle and not self.clients and not self.pending:
                    break
        finally:
            sel.close()
            srv.close()
            try:
                os.unlink(self.socket_path)
            except FileNotFoundError:
                pass
            for f in self.files:
                if f.fd >= 0:
                    os.close(f.fd)
        return rc

    def _handle(self, sel, conn: socket.socket, stop: dict) -> bool:
        try:
            data = conn.recv(MAX_MESSAGE)
        except OSError:
            data = b""
        if not data:  # a client left: its lease ends
            sel.unregister(conn)
            self.clients.pop(conn.fileno(), None)
            self.pending = [(c, m) for c, m in self.pending if c is not conn]
            conn.close()
            return False
        msg = json.loads(data.decode())
        op = msg.get("op")
        if op == "status":
            _send(conn, self.status())
        elif op == "release":
            mode = msg.get("mode", "drain")
            if mode not in ("idle", "drain", "force"):
                _send(conn, {"ok": False, "error": f"unknown mode {mode}"})
                return False
            exits = mode == "force" or not self.clients
            if mode == "idle" and self.clients:
                _send(conn, {"ok": True, "exits": False})
                return False
            if mode == "drain":
                self.exit_when_idle = True
                with self._lock:
                    self.state = "draining" if self.clients else self.state
            _send(conn, {"ok": True, "exits": exits})
            if exits:
                stop["now"] = True
                return True
        elif op == "attach":
            if self.exit_when_idle:
                _send(conn, {"ok": False, "error": "draining: no new attaches"})
            elif self._done.is_set() and self.state == "ready":
                answer, fds = self._attach_answer(msg)
                _send(conn, answer, fds)
                if answer["ok"]:
                    self.clients[conn.fileno()] = conn
            else:
                self.pending.append((conn, msg))  # answered once the fill is done
        else:
            _send(conn, {"ok": False, "error": f"unknown op {op}"})
        return False


class Attachment:
    """A client's lease on held files: read-only descriptors, kept until `close()`."""

    def __init__(self, socket_path: str, paths: list[str], timeout: float | None = None):
        self.sock = _connect(socket_path, timeout)
        idents = [file_identity(p) for p in paths]
        _send(self.sock, {"op": "attach", "files": idents})
        answer, fds = _recv(self.sock, maxfds=len(paths))
        if not answer.get("ok"):
            self.sock.close()
            raise SegmentError(answer.get("error", "attach refused"))
        self.manifest = answer["manifest"]
        self.fds = {os.path.basename(p): fd for p, fd in zip(paths, fds)}
        self.sizes = {os.path.basename(i["path"]): i["size"] for i in idents}

    def fd_path(self, path: str) -> str:
        return f"/proc/self/fd/{self.fds[os.path.basename(path)]}"

    def map(self, path: str, offset: int, nbytes: int) -> tuple[mmap.mmap, int]:
        """Read-only mapping of bytes [offset, offset + nbytes) of a held file, populated now.
        Returns the mapping and the position of `offset` inside it (mappings start on pages)."""
        name = os.path.basename(path)
        if offset < 0 or offset + nbytes > self.sizes[name]:
            raise SegmentError("range outside the file")
        start = offset - offset % mmap.ALLOCATIONGRANULARITY
        flags = mmap.MAP_SHARED | getattr(mmap, "MAP_POPULATE", 0)
        m = mmap.mmap(self.fds[name], nbytes + (offset - start), flags=flags, prot=mmap.PROT_READ, offset=start)
        return m, offset - start

    def close(self) -> None:
        for fd in self.fds.values():
            os.close(fd)
        self.fds = {}
        self.sock.close()


def _parse_file(v: str) -> tuple[str, str]:
    path, _, digest = v.rpartition("=")
    if not path or len(digest) != 64:
        raise argparse.ArgumentTypeError("--file takes PATH=SHA256")
    return path, digest


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="hold table files in sealed memory across server restarts")
    sub = ap.add_subparsers(dest="cmd", required=True)
    h = sub.add_parser("hold")
    h.add_argument("--socket", required=True)
    h.add_argument("--label", required=True)
    h.add_argument("--file", action="append", type=_parse_file, required=True)
    h.add_argument("--readers", type=int, default=1, help="accepted for launch-script compatibility; one reader")
    st = sub.add_parser("status")
    st.add_argument("--socket", required=True)
    rl = sub.add_parser("release")
    rl.add_argument("--socket", required=True)
    rl.add_argument("--mode", default="drain", choices=["idle", "drain", "force"])
    a = ap.parse_args(argv)
    if a.cmd == "hold":
        return Holder(a.socket, a.label, a.file).serve()
    print(json.dumps(request(a.socket, {"op": a.cmd} if a.cmd == "status" else {"op": "release", "mode": a.mode})))
    return 0


if __name__ == "__main__":
    sys.exit(main())
