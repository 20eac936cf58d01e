"""Load side: GGUF tensor bytes from a file into HBM, kept in their block format.

The reference uploads every tensor through WeightLoader._roh (ggufengine/models/common.py:83-116): the
file is read in 32 MiB pieces into a ring of 4 pinned buffers, each piece copied to the device on a
copy stream while the next one is read, the compute stream waiting on the copy stream at the end.
`Uploader.roh(gg, ti)` does the same job with the same inputs (any reader with `read_into(ti, out,
start)` and TensorInfo-like descriptors: the reference's gguf.GGUFFile, or `GGUFReader` below) and one
difference in how the overlap is made: a reader thread fills the pinned ring ahead of the copies (file
reads release the GIL), so the file is read at its own speed while earlier pieces cross PCIe, instead of
each read waiting for the host to reach it.  `install(loader)` puts it in place of a reference
WeightLoader's `_roh`.

`GGUFReader` / `write_gguf` are a small reader and writer of GGUF v2/v3 (header, typed metadata, tensor
descriptors, aligned data section; the public file layout) for fixtures and for use without the
reference: every count, length and extent read from a file is checked against limits and the file size
before use, as the reference's reader does (ggufengine/gguf.py:203-271).
"""
from __future__ import annotations

import mmap
import os
import queue
import struct
import threading
from dataclasses import dataclass
from typing import Any, Dict, Iterable, List, Optional, Sequence, Tuple

import torch

from .formats import GGML_TYPES

GGUF_MAGIC = b"GGUF"
MAX_TENSORS = 1 << 18
MAX_KV = 1 << 16
MAX_STRING = 16 << 20
MAX_ARRAY = 1 << 24
MAX_DIMS = 5
DEFAULT_ALIGNMENT = 32

(T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL,
 T_STRING, T_ARRAY, T_UINT64, T_INT64, T_FLOAT64) = range(13)
_SCALAR = {T_UINT8: "B", T_INT8: "b", T_UINT16: "H", T_INT16: "h", T_UINT32: "I", T_INT32: "i",
           T_FLOAT32: "f", T_BOOL: "?", T_UINT64: "Q", T_INT64: "q", T_FLOAT64: "d"}


class GGUFError(ValueError):
    """A malformed or out-of-bounds GGUF file."""


@dataclass(frozen=True)
class TensorInfo:
    """One tensor descriptor; the attribute names of the reference's gguf.TensorInfo."""
    name: str
    dims: Tuple[int, ...]           # GGUF order: dims[0] varies fastest
    ggml_type: int
    offset: int                     # from the start of the data section
    n_elements: int
    n_bytes: int

    @property
    def shape(self) -> Tuple[int, ...]:
        return tuple(reversed(self.dims))

    @property
    def type_name(self) -> str:
        return GGML_TYPES[self.ggml_type][0]


def tensor_nbytes(ggml_type: int, dims: Sequence[int]) -> int:
    """Bytes of a tensor: whole blocks along dims[0] (one element per block for the dense types)."""
    if ggml_type not in GGML_TYPES:
        raise GGUFError(f"unknown tensor type {ggml_type}")
    name, bv, bb = GGML_TYPES[ggml_type]
    n = 1
    for d in dims:
        n *= int(d)
    if int(dims[0]) % bv:
        raise GGUFError(f"{name}: row of {dims[0]} values is not whole blocks of {bv}")
    return n // bv * bb


class _Cursor:
    def __init__(self, buf, end: int):
        self.buf, self.pos, self.end = buf, 0, end

    def raw(self, n: int) -> bytes:
        if n < 0 or self.pos + n > self.end:
            raise GGUFError("truncated header")
        b = bytes(self.buf[self.pos:self.pos + n])
        self.pos += n
        return b

    def scalar(self, t: int):
        fmt = "<" + _SCALAR[t]
        return struct.unpack(fmt, self.raw(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.scalar(T_UINT64)
        if n > MAX_STRING:
            raise GGUFError(f"string of {n} bytes")
        return self.raw(n).decode("utf-8")

    def value(self, t: int, depth: int = 0):
        if t in _SCALAR:
            return self.scalar(t)
        if t == T_STRING:
            return self.string()
        if t == T_ARRAY and depth == 0:
            et = self.scalar(T_UINT32)
            n = self.scalar(T_UINT64)
            if n > MAX_ARRAY:
                raise GGUFError(f"array of {n} elements")
            return [self.value(et, 1) for _ in range(n)]
        raise GGUFError(f"bad metadata type {t}")


class GGUFReader:
    """Read-only GGUF file: metadata dict, tensors by name, zero-copy byte views and plain reads."""

    def __init__(self, path):
        self.path = os.fspath(path)
        self._fh = open(self.path, "rb")
        self.file_size = os.fstat(self._fh.fileno()).st_size
        self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ) if self.file_size else b""
        self._lock = threading.Lock()
        self.metadata: Dict[str, Any] = {}
        self.tensors: Dict[str, TensorInfo] = {}
        self.tensor_list: List[TensorInfo] = []
        self._parse()

    def _parse(self) -> None:
        c = _Cursor(self._mm, self.file_size)
        if c.raw(4) != GGUF_MAGIC:
            raise GGUFError("bad magic (not a GGUF file)")
        self.version = c.scalar(T_UINT32)
        if self.version not in (2, 3):
            raise GGUFError(f"unsupported GGUF version {self.version}")
        n_tensors, n_kv = c.scalar(T_UINT64), c.scalar(T_UINT64)
        if n_tensors > MAX_TENSORS or n_kv > MAX_KV:
            raise GGUFError(f"{n_tensors} tensors / {n_kv} metadata entries")
        for _ in range(n_kv):
            key = c.string()
            if not key or key in self.metadata:
                raise GGUFError(f"empty or duplicate metadata key {key!r}")
            self.metadata[key] = c.value(c.scalar(T_UINT32))
        align = self.metadata.get("general.alignment", DEFAULT_ALIGNMENT)
        if not isinstance(align, int) or isinstance(align, bool) or not 8 <= align <= 1 << 16 or align & (align - 1):
            raise GGUFError(f"invalid general.alignment {align!r}")
        self.alignment = align
        infos = []
        for _ in range(n_tensors):
            name = c.string()
            nd = c.scalar(T_UINT32)
            if not name or not 1 <= nd <= MAX_DIMS:
                raise GGUFError(f"tensor {name!r}: {nd} dims")
            dims = tuple(c.scalar(T_UINT64) for _ in range(nd))
            t = c.scalar(T_UINT32)
            off = c.scalar(T_UINT64)
            n_el = 1
            for d in dims:
                n_el *= d
            infos.append(TensorInfo(name, dims, t, off, n_el, tensor_nbytes(t, dims)))
        self.data_offset = (c.pos + align - 1) // align * align
        if self.data_offset > self.file_size:
            raise GGUFError("data section starts beyond the end of the file")
        data_size = self.file_size - self.data_offset
        end = 0
        for ti in sorted(infos, key=lambda x: x.offset):
            if ti.name in self.tensors:
                raise GGUFError(f"duplicate tensor {ti.name!r}")
            if ti.offset % align or ti.offset < end or ti.offset > data_size or ti.n_bytes > data_size - ti.offset:
                raise GGUFError(f"tensor {ti.name!r}: offset {ti.offset}, {ti.n_bytes} bytes outside the data")
            end = ti.offset + ti.n_bytes
            self.tensors[ti.name] = ti
        self.tensor_list = infos

    def tensor_bytes(self, ti: TensorInfo) -> memoryview:
        start = self.data_offset + ti.offset
        return memoryview(self._mm)[start:start + ti.n_bytes]

    def read_into(self, ti: TensorInfo, out, start: int = 0) -> int:
        """Bytes [start, start + len(out)) of the tensor into the writable buffer `out` with plain file
        reads; stops at the tensor's end and returns the count."""
        view = memoryview(out).cast("B")
        if not 0 <= start <= ti.n_bytes:
            raise GGUFError("read outside the tensor")
        n = min(view.nbytes, ti.n_bytes - start)
        with self._lock:
            self._fh.seek(self.data_offset + ti.offset + start)
            got = 0
            while got < n:
                k = self._fh.readinto(view[got:n])
                if not k:
                    raise GGUFError("unexpected end of file")
                got += k
        return n

    def close(self) -> None:
        if isinstance(self._mm, mmap.mmap):
            try:
                self._mm.close()
            except BufferError:
                pass
        self._fh.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def write_gguf(path, tensors: Iterable[Tuple[str, Sequence[int], int, bytes]], metadata: Optional[dict] = None,
               alignment: int = DEFAULT_ALIGNMENT) -> None:
    """GGUF v3 with string / int / float metadata and tensors (name, dims in GGUF order, ggml type, raw
    bytes), each tensor at an aligned offset."""
    tensors = list(tensors)
    meta = dict(metadata or {})
    if alignment != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = alignment

    def s(x: str) -> bytes:
        b = x.encode("utf-8")
        return struct.pack("<Q", len(b)) + b
    head = bytearray(GGUF_MAGIC + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for k, v in meta.items():
        head += s(k)
        if isinstance(v, str):
            head += struct.pack("<I", T_STRING) + s(v)
        elif isinstance(v, bool):
            head += struct.pack("<I?", T_BOOL, v)
        elif isinstance(v, int):
            head += struct.pack("<Iq" if v < 0 else "<IQ", T_INT64 if v < 0 else T_UINT64, v) if abs(v) >= 1 << 31 \
                else struct.pack("<Ii" if v < 0 else "<II", T_INT32 if v < 0 else T_UINT32, v)
        elif isinstance(v, float):
            head += struct.pack("<If", T_FLOAT32, v)
        else:
            raise TypeError(f"metadata {k}: {type(v).__name__}")
    off = 0
    offsets = []
    for name, dims, t, data in tensors:
        if len(data) != tensor_nbytes(t, dims):
            raise ValueError(f"{name}: {len(data)} bytes for dims {tuple(dims)} of type {t}")
        offsets.append(off)
        head += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", t, off)
        off = (off + len(data) + alignment - 1) // alignment * alignment
    pad = (-len(head)) % alignment
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        pos = 0
        for (name, dims, t, data), o in zip(tensors, offsets):
            f.write(b"\0" * (o - pos))
            f.write(data)
            pos = o + len(data)


class Uploader:
    """Raw tensor bytes into HBM through a ring of pinned buffers (the reference's WeightLoader._roh),
    read ahead by a thread.  One uploader per device; calls are serialised."""

    PIECE = 32 * 2 ** 20
    BUFFERS = 4

    def __init__(self, device, piece: int = PIECE, buffers: int = BUFFERS):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("Uploader: a CUDA device")
        if piece <= 0 or buffers < 2:
            raise ValueError("Uploader: piece > 0 and at least two buffers")
        self.piece = piece
        self.ring = [torch.empty(piece, dtype=torch.uint8, pin_memory=True) for _ in range(buffers)]
        self.done = [None] * buffers                 # event of the last copy out of each buffer
        self.stream = torch.cuda.Stream(self.device)
        self.loaded_bytes = 0
        self._lock = threading.Lock()

    def roh(self, gg, ti) -> torch.Tensor:
        """ti's bytes as a new uint8 tensor on the device; the current stream waits for the copies."""
        with self._lock:
            dst = torch.empty(ti.n_bytes, dtype=torch.uint8, device=self.device)
            # dst may reuse memory that kernels queued on the compute stream still read
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
            starts = list(range(0, ti.n_bytes, self.piece))
            # a buffer goes back to the reader only with the event of the copy that last read it
            free: "queue.Queue" = queue.Queue()
            for b, ev in enumerate(self.done):
                free.put((b, ev))
            filled: "queue.Queue" = queue.Queue()
            err: List[BaseException] = []

            def reader():
                try:
                    for start in starts:
                        b, ev = free.get()
                        if ev is not None:
                            ev.synchronize()                     # its previous copy has left the buffer
                        n = gg.read_into(ti, self.ring[b].numpy(), start)
                        filled.put((b, start, n))
                except BaseException as e:                       # handed to the caller below
                    err.append(e)
                finally:
                    filled.put(None)
            th = threading.Thread(target=reader, daemon=True)
            th.start()
            with torch.cuda.stream(self.stream):
                while True:
                    item = filled.get()
                    if item is None:
                        break
                    b, start, n = item
                    dst[start:start + n].copy_(self.ring[b][:n], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(self.stream)
                    self.done[b] = ev
                    free.put((b, ev))
            th.join()
            if err:
                raise err[0]
            dst.record_stream(self.stream)
            torch.cuda.current_stream(self.device).wait_stream(self.stream)
            self.loaded_bytes += ti.n_bytes
            return dst


def install(loader, **kw) -> Uploader:
    """Replace a reference WeightLoader's `_roh(ti, device)` on a CUDA device by Uploader.roh (CPU
    targets keep the loader's own path)."""
    up = Uploader(loader.device, **kw)
    own = loader._roh

    def _roh(ti, device):
        device = torch.device(device)
        if device.type != "cuda":
            return own(ti, device)
        return up.roh(loader.gg, ti)
    loader._roh = _roh
    return up
