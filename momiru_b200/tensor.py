"""Device storage and strided views for the matmul hot path.

Mirrors the reference's host tensor model for device memory:
  * `DeviceBuffer` ~ BufferHandle::Device{device_ordinal, address, bytes}
    (src/momiru/tensor_light/execution/runtime.rs:297-301), plus an allocation
    identity so the binder can prove an output disjoint from its inputs.
  * `DeviceView` ~ Shape{dims, strides} over a storage with a base offset
    (tensor/shape.rs:130-206, TensorStoragePlan plan.rs:1285-1307), with the
    zero-copy view operations `transpose`, `narrow`, `slice` and
    `as_strided_view` of TensorView (tensor/view.rs:450, 791, 800, 488).
Device memory is allocated through torch (plumbing only); compute never goes
through torch.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass, field

import numpy as np

from . import _abi

_alloc_ids = itertools.count(1)


class ViewError(ValueError):
    pass


@dataclass
class DeviceBuffer:
    """A device allocation (or a raw external handle) the caller owns."""
    address: int
    bytes: int
    device_ordinal: int = 0
    allocation_id: int = field(default_factory=lambda: next(_alloc_ids))
    owner: object = None  # keeps a torch tensor alive when we allocated it

    @staticmethod
    def allocate(nbytes: int, device_ordinal: int = 0) -> "DeviceBuffer":
        import torch
        n = max(1, (nbytes + 3) // 4)
        t = torch.empty(n, dtype=torch.float32, device=f"cuda:{device_ordinal}")
        return DeviceBuffer(t.data_ptr(), n * 4, device_ordinal, owner=t)

    @staticmethod
    def from_torch(t) -> "DeviceBuffer":
        """Borrow the storage of a CUDA torch tensor (no copy)."""
        st = t.untyped_storage()
        return DeviceBuffer(st.data_ptr(), st.nbytes(), t.device.index or 0, owner=t)


@dataclass(frozen=True)
class DeviceView:
    buffer: DeviceBuffer
    dims: tuple
    strides: tuple          # element strides (>= 0)
    offset: int = 0         # element offset of [0, .., 0]

    # ---------------------------------------------------------------- create
    @staticmethod
    def contiguous(buffer: DeviceBuffer, dims, offset: int = 0) -> "DeviceView":
        dims = tuple(int(d) for d in dims)
        strides, acc = [], 1
        for d in reversed(dims):
            strides.append(acc)
            acc *= max(d, 1)
        return DeviceView(buffer, dims, tuple(reversed(strides)), offset)

    @staticmethod
    def empty(dims, device_ordinal: int = 0) -> "DeviceView":
        n = int(np.prod(dims)) if len(dims) else 1
        return DeviceView.contiguous(DeviceBuffer.allocate(4 * n, device_ordinal), dims)

    @staticmethod
    def from_host(arr: np.ndarray, device_ordinal: int = 0) -> "DeviceView":
        import torch
        a = np.ascontiguousarray(arr, dtype=np.float32)
        t = torch.from_numpy(a).to(f"cuda:{device_ordinal}")
        return DeviceView.contiguous(DeviceBuffer.from_torch(t), a.shape)

    # ------------------------------------------------------------ properties
    @property
    def rank(self) -> int:
        return len(self.dims)

    @property
    def numel(self) -> int:
        return int(np.prod(self.dims)) if self.dims else 1

    def is_row_major_contiguous(self) -> bool:
        return self == DeviceView.contiguous(self.buffer, self.dims, self.offset)

    # ------------------------------------------------------------ view ops
    def transpose(self, a: int = -2, b: int = -1) -> "DeviceView":
        a %= self.rank
        b %= self.rank
        d, s = list(self.dims), list(self.strides)
        d[a], d[b] = d[b], d[a]
        s[a], s[b] = s[b], s[a]
        return DeviceView(self.buffer, tuple(d), tuple(s), self.offset)

    def narrow(self, axis: int, start: int, length: int) -> "DeviceView":
        axis %= self.rank
        if start < 0 or length < 0 or start + length > self.dims[axis]:
            raise ViewError(f"narrow({axis}, {start}, {length}) outside extent {self.dims[axis]}")
        d = list(self.dims)
        d[axis] = length
        return DeviceView(self.buffer, tuple(d), self.strides, self.offset + start * self.strides[axis])

    def slice(self, specs) -> "DeviceView":
        """specs: one (start, stop, step>0) tuple or None (full axis) per axis."""
        d, s, off = list(self.dims), list(self.strides), self.offset
        for ax, spec in enumerate(specs):
            if spec is None:
                continue
            start, stop, step = spec
            if step <= 0 or not (0 <= start <= stop <= self.dims[ax]):
                raise ViewError(f"slice spec {spec} invalid for axis {ax}")
            off += start * s[ax]
            d[ax] = (stop - start + step - 1) // step
            s[ax] *= step
        return DeviceView(self.buffer, tuple(d), tuple(s), off)

    def as_strided_view(self, dims, strides, offset: int | None = None) -> "DeviceView":
        return DeviceView(self.buffer, tuple(dims), tuple(strides), self.offset if offset is None else offset)

    def unsqueeze(self, axis: int) -> "DeviceView":
        d, s = list(self.dims), list(self.strides)
        d.insert(axis, 1)
        s.insert(axis, 0)
        return DeviceView(self.buffer, tuple(d), tuple(s), self.offset)

    # ----------------------------------------------------------- host copies
    def torch_view(self):
        """A torch view over the same memory (for copies in and out)."""
        import torch
        base = self.buffer.owner
        if base is None or not isinstance(base, torch.Tensor) or base.dtype != torch.float32:
            raise ViewError("buffer not allocated through torch as f32")
        # as_strided offsets are absolute within the storage, as ours are.
        return torch.as_strided(base, self.dims, self.strides, self.offset)

    def to_host(self) -> np.ndarray:
        return self.torch_view().cpu().numpy()

    def copy_from_host(self, arr: np.ndarray) -> None:
        import torch
        self.torch_view().copy_(torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32)))

    # ------------------------------------------------------------------ ABI
    def to_abi(self) -> _abi.MmrView:
        if self.rank > _abi.MAX_RANK:
            raise ViewError(f"rank {self.rank} above {_abi.MAX_RANK}")
        v = _abi.MmrView()
        v.address = self.buffer.address
        v.bytes = self.buffer.bytes
        v.base_offset_bytes = 4 * self.offset
        v.rank = self.rank
        v.device_ordinal = self.buffer.device_ordinal
        for i, (d, s) in enumerate(zip(self.dims, self.strides)):
            v.dims[i] = d
            v.strides[i] = s
        v.allocation_id = self.buffer.allocation_id
        return v
