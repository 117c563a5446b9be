"""GGUF model files: the on-disk source of k-quant weights, read through libkq.so's reader
(``kq_gguf_*`` in include/kq.h; host code, no GPU needed).

A GGUF tensor stores a matrix exactly as ``kq_matvec`` takes it: ``shape`` is GGUF's dimension
order (``shape[0]`` = k elements per row, ``shape[1]`` = rows) and the bytes are the rows back to
back, so a Q4_K / Q5_K / Q6_K tensor goes to the device as it is::

    with GGUFFile("model.gguf") as f:
        t = f.tensor("blk.0.attn_q.weight")
        W = t.to_device()                        # torch uint8 on the current GPU
        kernels.matvec(t.qtype, y, W, x, t.rows, t.k)
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import Error, KqGgufTensor, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K, _check, lib

# GGML type numbers the library's matvec takes, by name
QTYPES = {TYPE_Q4_K: 4, TYPE_Q5_K: 5, TYPE_Q6_K: 6}


@dataclass
class Tensor:
    """One tensor of a GGUF file; ``data`` is a read-only view of the mapped file (valid while
    the file is open)."""

    name: str
    type: int          # GGML type number (12 = Q4_K, 13 = Q5_K, 14 = Q6_K, 0 = F32, ...)
    shape: tuple       # GGUF order: shape[0] innermost
    offset: int        # byte offset of the data in the file
    data: np.ndarray   # uint8 view; empty when the reader does not know the type's block size

    @property
    def qtype(self) -> int:
        """4, 5 or 6 for a Q4_K / Q5_K / Q6_K tensor kq_matvec can multiply, else raises."""
        if self.type not in QTYPES:
            raise Error("gguf", f"tensor {self.name} has GGML type {self.type}, not Q4_K/Q5_K/Q6_K")
        return QTYPES[self.type]

    @property
    def k(self) -> int:
        return int(self.shape[0])

    @property
    def rows(self) -> int:
        return int(np.prod(self.shape[1:], dtype=np.int64)) if len(self.shape) > 1 else 1

    def to_device(self, device=None):
        """The tensor's bytes in a new torch uint8 tensor on the GPU (one host-to-device copy)."""
        import torch

        return torch.from_numpy(np.array(self.data, copy=True)).to(device or "cuda")


class GGUFFile:
    """A mapped GGUF file (``kq_gguf_open``); close it, or use it as a context manager."""

    def __init__(self, path: str):
        self._h = ctypes.c_void_p()
        _check(lib().kq_gguf_open(str(path).encode(), ctypes.byref(self._h)), "kq_gguf_open")

    def close(self) -> None:
        if self._h:
            lib().kq_gguf_close(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self) -> "GGUFFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return int(lib().kq_gguf_tensor_count(self._h))

    def _wrap(self, t: KqGgufTensor) -> Tensor:
        n = int(t.nbytes)
        if n:
            buf = (ctypes.c_uint8 * n).from_address(t.data)
            data = np.frombuffer(buf, dtype=np.uint8)
            data.flags.writeable = False
        else:
            data = np.empty(0, dtype=np.uint8)
        return Tensor(name=t.name.decode(), type=int(t.type),
                      shape=tuple(int(t.dims[i]) for i in range(t.n_dims)),
                      offset=int(t.offset), data=data)

    def tensors(self) -> list[Tensor]:
        out = []
        for i in range(len(self)):
            t = KqGgufTensor()
            _check(lib().kq_gguf_tensor_at(self._h, i, ctypes.byref(t)), "kq_gguf_tensor_at")
            out.append(self._wrap(t))
        return out

    def tensor(self, name: str) -> Tensor:
        t = KqGgufTensor()
        _check(lib().kq_gguf_find(self._h, name.encode(), ctypes.byref(t)), "kq_gguf_find")
        return self._wrap(t)

    def meta_int(self, key: str) -> int:
        v = ctypes.c_int64()
        _check(lib().kq_gguf_meta_int(self._h, key.encode(), ctypes.byref(v)), "kq_gguf_meta_int")
        return int(v.value)

    def meta_str(self, key: str) -> str:
        v = ctypes.c_char_p()
        _check(lib().kq_gguf_meta_str(self._h, key.encode(), ctypes.byref(v)), "kq_gguf_meta_str")
        return v.value.decode()
