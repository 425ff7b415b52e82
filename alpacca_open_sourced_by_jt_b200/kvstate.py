"""Device-authoritative KV state of attention layers, in the reference's
snapshot format, and a device mirror of a host f32 cache.

The reference keeps every layer's K/V rows on the host in f32: as flat
arrays behind FullAttentionState (alpaccaroo/memory.py:385-475), whose
snapshots are f32 little-endian byte strings (FullAttentionSnapshot,
memory.py:224-241); and as model.cache_k/cache_v, which the GPU decode
chain mirrors to the device (f32 or f16), tracking the mirrored prefix with
valid_upto and re-uploading from the first row a host mutation touched
(Model._chain_invalidate, model.py:966-978; DecodeChain.invalidate and
_sync_mirror, cuda.py:1875-1900; rows computed on the device come home
widened to f32, cuda.py:2046-2061).

On the B200 the 16-bit device cache is the authoritative copy:

* DeviceAttentionState keeps one layer's rows in a preallocated
  (n_ctx, kv_heads, dim) f32/f16/bf16 device buffer with the reference's
  state API (append, reset, truncate, clone, snapshot, restore,
  memory_bytes, describe).  A snapshot widens the live rows to f32 on the
  device and copies them to host bytes in the reference's record format, so
  a snapshot taken here restores into the reference and vice versa.
* DeviceMirror keeps the reference's arrangement (host f32 authoritative)
  for callers that need it: valid_upto, invalidate, sync (narrowing on the
  device) and fetch (widening on the device).

All conversions run through b2a_kv_convert; nothing here converts on the
host or falls back to the CPU.
"""
from __future__ import annotations

import sys
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

F32_LE = "f32-le"
_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


class StateError(ValueError):
    """Invalid state operation or record (the reference's memory.StateError)."""


class SnapshotMismatchError(StateError):
    """A snapshot that does not fit the layer it is restored into."""


@dataclass(frozen=True)
class AttentionSnapshot:
    """One attention layer's rows [0, logical_length) as f32 little-endian
    bytes, [row][kv_head][dim] order; the fields, their order and meaning
    follow FullAttentionSnapshot (alpaccaroo/memory.py:224-241)."""

    layer_index: int
    logical_length: int
    kv_heads: int
    key_dim: int
    value_dim: int
    key: bytes
    value: bytes
    dtype: str = F32_LE
    kind: str = "attention"

    def memory_bytes(self) -> int:
        return len(self.key) + len(self.value)


def convert(src: torch.Tensor, dst: torch.Tensor, stream=None) -> torch.Tensor:
    """dst[:] = src converted to dst's dtype, on the device (b2a_kv_convert:
    exact widening, round-to-nearest-even narrowing).  Both contiguous CUDA
    tensors with the same number of elements."""
    if not (src.is_cuda and dst.is_cuda and src.is_contiguous() and dst.is_contiguous()):
        raise _lib.B2AShapeError(_lib.ERR_SHAPE, "convert: contiguous CUDA tensors")
    if src.numel() != dst.numel():
        raise _lib.B2AShapeError(_lib.ERR_SHAPE, "convert: element counts differ")
    for t in (src, dst):
        if t.dtype not in _DT:
            raise _lib.B2AShapeError(_lib.ERR_DTYPE, f"convert: unsupported dtype {t.dtype}")
    if stream is None:
        stream = torch.cuda.current_stream(src.device).cuda_stream
    _lib.check(_lib.load().b2a_kv_convert(src.data_ptr(), _DT[src.dtype], dst.data_ptr(),
                                          _DT[dst.dtype], src.numel(), stream))
    return dst


def validate_snapshot(snap, *, layer_index: int, kv_heads: int, key_dim: int,
                      value_dim: int, capacity: int) -> None:
    """The reference's checks for an attention-layer record
    (alpaccaroo/memory.py:634-690: index, kind, record type, dtype, shape,
    payload sizes), plus the device buffer's row capacity."""
    if getattr(snap, "layer_index", None) != layer_index:
        raise SnapshotMismatchError(f"snapshot layer index mismatch at layer {layer_index}")
    if getattr(snap, "kind", None) != "attention":
        raise SnapshotMismatchError(f"snapshot layer {layer_index} kind differs from descriptor")
    for name in ("logical_length", "kv_heads", "key_dim", "value_dim", "key", "value", "dtype"):
        if not hasattr(snap, name):
            raise SnapshotMismatchError(f"snapshot layer {layer_index} has the wrong record type")
    if snap.dtype != F32_LE:
        raise SnapshotMismatchError(
            f"snapshot layer {layer_index} has unsupported dtype {snap.dtype!r}")
    if (snap.kv_heads != kv_heads or snap.key_dim != key_dim or snap.value_dim != value_dim
            or snap.logical_length < 0):
        raise SnapshotMismatchError(f"snapshot layer {layer_index} attention shape/position differs")
    if snap.logical_length > capacity:
        raise SnapshotMismatchError(
            f"snapshot layer {layer_index} holds {snap.logical_length} rows, capacity {capacity}")
    for what, data, dim in (("key", snap.key, key_dim), ("value", snap.value, value_dim)):
        if not isinstance(data, (bytes, bytearray, memoryview)):
            raise StateError(f"snapshot layer {layer_index} {what} payload must be bytes")
        want = snap.logical_length * kv_heads * dim * 4
        if len(data) != want:
            raise StateError(
                f"snapshot layer {layer_index} {what} has {len(data)} bytes, expected {want}")


class DeviceAttentionState:
    """One attention layer's K/V rows on the device: rows [0, logical_length)
    of a (n_ctx, kv_heads, key_dim|value_dim) buffer of `dtype`.  Appends
    normally happen in the fused RoPE + append kernel (pass .key/.value as
    its caches and advance with advance()); append() is the reference's
    one-row host API."""

    def __init__(self, layer_index: int, kv_heads: int, key_dim: int, value_dim: int,
                 n_ctx: int, dtype: torch.dtype = torch.bfloat16, device=None):
        if dtype not in _DT:
            raise StateError(f"unsupported cache dtype {dtype}")
        for name, v in (("kv_heads", kv_heads), ("key_dim", key_dim),
                        ("value_dim", value_dim), ("n_ctx", n_ctx)):
            if int(v) <= 0:
                raise StateError(f"{name} must be positive, got {v}")
        if int(layer_index) < 0:
            raise StateError(f"layer_index must be non-negative, got {layer_index}")
        _lib.load()
        self.layer_index, self.kv_heads = int(layer_index), int(kv_heads)
        self.key_dim, self.value_dim, self.n_ctx = int(key_dim), int(value_dim), int(n_ctx)
        self.dtype = dtype
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.key = torch.zeros((n_ctx, kv_heads, key_dim), dtype=dtype, device=self.device)
        self.value = torch.zeros((n_ctx, kv_heads, value_dim), dtype=dtype, device=self.device)
        self.logical_length = 0
        self._pinned = torch.empty(0, dtype=torch.float32)  # grow-only snapshot staging

    @property
    def key_row_size(self) -> int:
        return self.kv_heads * self.key_dim

    @property
    def value_row_size(self) -> int:
        return self.kv_heads * self.value_dim

    def _rows_f32(self, data, row_size: int, what: str) -> torch.Tensor:
        a = np.asarray(data, dtype=np.float32).reshape(-1)
        if a.size % row_size:
            raise StateError(f"attention {what} has {a.size} float32 values, expected a "
                             f"multiple of {row_size}")
        return torch.from_numpy(a).to(self.device)

    def append(self, key, value) -> None:
        """Append one row (kv_heads * dim f32 values each), narrowed on the device."""
        k = self._rows_f32(key, self.key_row_size, "key row")
        v = self._rows_f32(value, self.value_row_size, "value row")
        if k.numel() != self.key_row_size or v.numel() != self.value_row_size:
            raise StateError("attention rows must hold exactly one row each")
        self.write_rows(self.logical_length, k, v)
        self.logical_length += 1

    def write_rows(self, start: int, key_f32: torch.Tensor, value_f32: torch.Tensor) -> None:
        """Rows [start, start + n) from f32 device or host rows (narrowed on
        the device); does not move logical_length."""
        k = key_f32.to(self.device, torch.float32).contiguous().reshape(-1)
        v = value_f32.to(self.device, torch.float32).contiguous().reshape(-1)
        n = k.numel() // self.key_row_size
        if (k.numel() != n * self.key_row_size or v.numel() != n * self.value_row_size
                or start < 0 or start + n > self.n_ctx):
            raise StateError(f"rows [{start}, {start + n}) do not fit capacity {self.n_ctx}")
        convert(k, self.key[start:start + n].reshape(-1))
        convert(v, self.value[start:start + n].reshape(-1))

    def advance(self, rows: int = 1) -> None:
        """Account for rows the append kernels wrote at logical_length.."""
        if rows < 0 or self.logical_length + rows > self.n_ctx:
            raise StateError(f"cannot advance {self.logical_length} by {rows} (capacity {self.n_ctx})")
        self.logical_length += rows

    def reset(self) -> None:
        self.logical_length = 0

    def truncate(self, position: int) -> None:
        """Keep rows [0, position) (memory.py:435-443: never extends)."""
        if position < 0:
            raise StateError(f"position must be non-negative, got {position}")
        if position > self.logical_length:
            raise StateError(
                f"cannot extend attention state from {self.logical_length} to {position}")
        self.logical_length = int(position)

    def clone(self) -> "DeviceAttentionState":
        c = DeviceAttentionState(self.layer_index, self.kv_heads, self.key_dim, self.value_dim,
                                 self.n_ctx, self.dtype, self.device)
        n = self.logical_length
        c.key[:n].copy_(self.key[:n])
        c.value[:n].copy_(self.value[:n])
        c.logical_length = n
        return c

    def _host_bytes(self, rows: torch.Tensor, count: int) -> bytes:
        """rows (16-bit or f32, on the device) widened to f32 on the device,
        copied into pinned staging, returned as little-endian bytes."""
        if count == 0:
            return b""
        if self._pinned.numel() < count:
            self._pinned = torch.empty(count, dtype=torch.float32).pin_memory()
        f32 = torch.empty(count, dtype=torch.float32, device=self.device)
        convert(rows.reshape(-1), f32)
        host = self._pinned[:count]
        host.copy_(f32, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        a = host.numpy()
        return a.tobytes() if sys.byteorder == "little" else a.byteswap().tobytes()

    def snapshot(self) -> AttentionSnapshot:
        """The live rows widened to f32 on the device, as the reference's record."""
        n = self.logical_length
        return AttentionSnapshot(
            layer_index=self.layer_index, logical_length=n, kv_heads=self.kv_heads,
            key_dim=self.key_dim, value_dim=self.value_dim,
            key=self._host_bytes(self.key[:n], n * self.key_row_size),
            value=self._host_bytes(self.value[:n], n * self.value_row_size))

    def restore(self, snap) -> None:
        """Validate, then load a snapshot's rows (narrowed on the device).
        Accepts this module's records and the reference's
        FullAttentionSnapshot alike."""
        validate_snapshot(snap, layer_index=self.layer_index, kv_heads=self.kv_heads,
                          key_dim=self.key_dim, value_dim=self.value_dim, capacity=self.n_ctx)
        n = snap.logical_length
        if n:
            order = "<f4"
            k = np.frombuffer(bytes(snap.key), dtype=order).reshape(n, self.kv_heads, self.key_dim)
            v = np.frombuffer(bytes(snap.value), dtype=order).reshape(n, self.kv_heads,
                                                                       self.value_dim)
            self.write_rows(0, torch.from_numpy(k.astype(np.float32)),
                            torch.from_numpy(v.astype(np.float32)))
        self.logical_length = n

    @classmethod
    def from_snapshot(cls, snap, n_ctx: int, dtype: torch.dtype = torch.bfloat16,
                      device=None) -> "DeviceAttentionState":
        st = cls(snap.layer_index, snap.kv_heads, snap.key_dim, snap.value_dim, n_ctx, dtype,
                 device)
        st.restore(snap)
        return st

    def memory_bytes(self) -> int:
        """The reference's count: f32 bytes of the live rows (memory.py:462-463)."""
        return self.logical_length * (self.key_row_size + self.value_row_size) * 4

    def device_bytes(self) -> int:
        return self.key.numel() * self.key.element_size() + \
            self.value.numel() * self.value.element_size()

    def describe(self) -> dict:
        n = self.logical_length
        return {
            "kind": "attention", "layer_index": self.layer_index, "logical_length": n,
            "dtype": str(self.dtype).replace("torch.", ""),
            "key_shape": [n, self.kv_heads, self.key_dim],
            "value_shape": [n, self.kv_heads, self.value_dim],
            "memory_bytes": self.memory_bytes(), "device_bytes": self.device_bytes(),
            "capacity": self.n_ctx,
        }


class DeviceMirror:
    """A device copy (f32/f16/bf16) of a host-authoritative f32 KV cache,
    the arrangement of the reference's GPU decode chain: rows
    [0, valid_upto) on the device equal the host rows (rounded to the
    mirror dtype).  host_k/host_v: per-layer (n_ctx, kv_heads, head_dim)
    float32 NumPy arrays, which the caller keeps mutating."""

    def __init__(self, host_k, host_v, dtype: torch.dtype = torch.bfloat16, device=None):
        if len(host_k) != len(host_v) or not host_k:
            raise StateError("one K and one V array per layer")
        shape = host_k[0].shape
        for a in list(host_k) + list(host_v):
            if a.dtype != np.float32 or a.shape != shape or a.ndim != 3:
                raise StateError("host caches must be float32 (n_ctx, kv_heads, head_dim)")
        if dtype not in _DT:
            raise StateError(f"unsupported mirror dtype {dtype}")
        _lib.load()
        self.host_k, self.host_v = list(host_k), list(host_v)
        self.n_ctx = shape[0]
        self.row = shape[1] * shape[2]
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.k = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in host_k]
        self.v = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in host_v]
        self.valid_upto = 0
        self._stage = torch.empty(0, dtype=torch.float32).pin_memory()
        self._dstage = torch.empty(0, dtype=torch.float32, device=self.device)

    def _staging(self, n: int):
        if self._stage.numel() < n:
            self._stage = torch.empty(n, dtype=torch.float32).pin_memory()
            self._dstage = torch.empty(n, dtype=torch.float32, device=self.device)
        return self._stage[:n], self._dstage[:n]

    def invalidate(self, pos: int) -> None:
        """A host mutation touched rows from pos on (cuda.py:1875-1879)."""
        if pos < self.valid_upto:
            self.valid_upto = max(0, int(pos))

    def sync(self, upto: int) -> None:
        """Upload host rows [valid_upto, upto) of every layer, narrowed on
        the device (cuda.py:1881-1900)."""
        if upto < 0 or upto > self.n_ctx:
            raise StateError(f"sync bound {upto} outside [0, {self.n_ctx}]")
        a, b = self.valid_upto, int(upto)
        if b <= a:
            return
        n = (b - a) * self.row
        h, d = self._staging(n)
        hv = h.numpy()
        for layers, dev in ((self.host_k, self.k), (self.host_v, self.v)):
            for host, mirror in zip(layers, dev):
                hv[:] = host[a:b].reshape(-1)
                d.copy_(h, non_blocking=True)
                convert(d, mirror[a:b].reshape(-1))
                torch.cuda.current_stream(self.device).synchronize()  # staging reuse
        self.valid_upto = b

    def fetch(self, a: int, b: int) -> None:
        """Device rows [a, b) of every layer back into the host caches,
        widened on the device (rows computed on the device coming home,
        cuda.py:2046-2061)."""
        if not 0 <= a <= b <= self.n_ctx:
            raise StateError(f"fetch range [{a}, {b}) outside [0, {self.n_ctx}]")
        if b == a:
            return
        n = (b - a) * self.row
        h, d = self._staging(n)
        for layers, dev in ((self.host_k, self.k), (self.host_v, self.v)):
            for host, mirror in zip(layers, dev):
                convert(mirror[a:b].reshape(-1), d)
                h.copy_(d, non_blocking=True)
                torch.cuda.current_stream(self.device).synchronize()
                host[a:b] = h.numpy().reshape(b - a, *host.shape[1:])
