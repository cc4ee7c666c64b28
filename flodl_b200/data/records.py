"""Record files with a fixed byte stride per record, read one record at a time by offset.

Reference: flodl/src/data/records.rs. Many raw dataset files are fixed-size
records behind a fixed header (CIFAR-10 binary batches: 3073-byte records;
MNIST IDX images: 784-byte records behind a 16-byte header).
:class:`FixedStrideRecords` reads record ``i`` at ``header + i * stride``
with one positioned read (``pread``) and no shared seek state, so prefetch
and staging threads read concurrently without contention. A dataset built on
it reads storage per sample instead of loading the file - the path for data
larger than RAM; the loader's sample cache and disk stage compose on top.
"""
from __future__ import annotations

import os
from typing import Callable, List, Sequence

import numpy as np
import torch

from .loader import DataSet


class FixedStrideRecords:
    def __init__(self, path: str, stride: int, header: int = 0):
        if stride <= 0 or header < 0:
            raise ValueError("stride must be positive and header non-negative")
        self.path, self.stride, self.header = path, stride, header
        self.fd = os.open(path, os.O_RDONLY)
        size = os.fstat(self.fd).st_size - header
        if size < 0 or size % stride:
            os.close(self.fd)
            raise ValueError(f"{path}: {size} payload bytes are not a whole number of "
                             f"{stride}-byte records")
        self.n = size // stride

    def __len__(self) -> int:
        return self.n

    def record(self, i: int) -> bytes:
        if not 0 <= i < self.n:
            raise IndexError(f"record {i} of {self.n}")
        b = os.pread(self.fd, self.stride, self.header + i * self.stride)
        if len(b) != self.stride:
            raise OSError(f"{self.path}: short read at record {i}")
        return b

    def close(self) -> None:
        os.close(self.fd)

    def __del__(self):
        try:
            os.close(self.fd)
        except OSError:
            pass


class RecordDataSet(DataSet):
    """A per-sample dataset over one or more record files: ``parse(bytes) ->
    [tensors]`` turns a record into the sample."""

    def __init__(self, files: Sequence[FixedStrideRecords], parse: Callable[[bytes], List[torch.Tensor]]):
        self.files = list(files)
        self.parse = parse
        self.offsets = np.cumsum([0] + [len(f) for f in self.files])

    def __len__(self) -> int:
        return int(self.offsets[-1])

    def get(self, i: int) -> List[torch.Tensor]:
        k = int(np.searchsorted(self.offsets, i, side="right")) - 1
        return self.parse(self.files[k].record(i - int(self.offsets[k])))


_CIFAR_MEAN = np.array([0.4914, 0.4822, 0.4465], dtype=np.float32).reshape(3, 1, 1)
_CIFAR_STD = np.array([0.2470, 0.2435, 0.2616], dtype=np.float32).reshape(3, 1, 1)


def cifar10_records(root: str, train: bool = True) -> RecordDataSet:
    """CIFAR-10 binary batches read per record (label byte + 3x32x32 image)."""
    names = [f"data_batch_{i}.bin" for i in range(1, 6)] if train else ["test_batch.bin"]

    def parse(b: bytes):
        a = np.frombuffer(b, dtype=np.uint8)
        img = (a[1:].reshape(3, 32, 32).astype(np.float32) / 255.0 - _CIFAR_MEAN) / _CIFAR_STD
        return [torch.from_numpy(img), torch.tensor(int(a[0]), dtype=torch.int64)]

    return RecordDataSet([FixedStrideRecords(os.path.join(root, n), 3073) for n in names], parse)


def mnist_records(root: str, train: bool = True) -> RecordDataSet:
    """MNIST IDX images (16-byte header, 784-byte records) with their labels
    (8-byte header, 1-byte records), uncompressed files."""
    pre = "train" if train else "t10k"
    imgs = FixedStrideRecords(os.path.join(root, f"{pre}-images-idx3-ubyte"), 784, 16)
    labs = FixedStrideRecords(os.path.join(root, f"{pre}-labels-idx1-ubyte"), 1, 8)

    class _Mnist(DataSet):
        def __len__(self):
            return len(imgs)

        def get(self, i):
            x = np.frombuffer(imgs.record(i), dtype=np.uint8).astype(np.float32) / 255.0
            return [torch.from_numpy(x).view(1, 28, 28), torch.tensor(labs.record(i)[0], dtype=torch.int64)]

    return _Mnist()
