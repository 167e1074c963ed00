"""Nameless scratch files for NVMe offload (activations, optimizer state).

A ``ScratchFile`` lives in a directory but has no name: it is opened with
O_TMPFILE where the filesystem supports that, else created and unlinked at
once.  Its space is returned when the descriptor closes, including when the
process dies, so an interrupted run never leaves offload files behind (the
reference's offload files stay on disk after a crash).  Reads and writes are
positional (pread/pwrite), so different files can be used from several I/O
threads at once.
"""
from __future__ import annotations

import os
import tempfile

# one pread/pwrite moves at most this much on Linux
_CHUNK = 1 << 30


class ScratchFile:
    def __init__(self, directory: str):
        os.makedirs(directory, exist_ok=True)
        fd = -1
        tmpfile = getattr(os, "O_TMPFILE", 0)
        if tmpfile:
            try:
                fd = os.open(directory, tmpfile | os.O_RDWR, 0o600)
            except OSError:
                fd = -1
        if fd < 0:
            fd, path = tempfile.mkstemp(dir=directory, prefix="t1-scratch-")
            os.unlink(path)
        self.fd = fd

    def write(self, data: memoryview, offset: int = 0) -> None:
        data = memoryview(data).cast("B")
        done = 0
        while done < len(data):
            n = os.pwrite(self.fd, data[done:done + _CHUNK], offset + done)
            if n <= 0:
                raise OSError(f"pwrite returned {n}")
            done += n

    def read_into(self, out: memoryview, offset: int = 0) -> None:
        out = memoryview(out).cast("B")
        done = 0
        while done < len(out):
            n = os.preadv(self.fd, [out[done:done + _CHUNK]], offset + done)
            if n <= 0:
                raise OSError(f"short read from a scratch file ({done} of {len(out)} bytes)")
            done += n

    def close(self) -> None:
        if self.fd >= 0:
            os.close(self.fd)
            self.fd = -1

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
