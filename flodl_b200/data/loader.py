"""Datasets and the DataLoader (flodl/src/data/mod.rs:139-198, loader.rs:111-476).

* ``DataSet``: ``len()`` and ``get(index) -> list[Tensor]`` (pure, per sample).
* ``BatchDataSet``: ``get_batch(indices) -> list[Tensor]``.
* ``DataLoader.from_dataset(ds).batch_size(..).device(..).seed(..).shuffle(..)
  .prefetch(..).vram_max_usage(..).streaming().drop_last(..).build()``.

Two modes, as in floDl:

* **resident**: the whole dataset is materialised once as stacked tensors on
  the target device; an epoch is a device-side permutation and each batch an
  ``index_select`` on the GPU (no host traffic after the first load).
* **streaming**: batches are gathered on the host into pinned buffers by the
  native prefetch thread and copied to the device on a dedicated stream,
  ``depth`` batches ahead. Resident is chosen when the dataset fits in the
  VRAM budget (``vram_max_usage`` of free memory), streaming otherwise or when
  forced; an out-of-memory error during the resident load falls back to
  streaming.
"""
from __future__ import annotations

import math
from typing import Callable, Iterator, List, Optional, Sequence

import torch

from .sampler import RandomSampler, Sampler, SequentialSampler


class DataSet:
    def __len__(self) -> int:  # pragma: no cover - interface
        raise NotImplementedError

    def len(self) -> int:
        return len(self)

    def get(self, index: int) -> List[torch.Tensor]:  # pragma: no cover - interface
        raise NotImplementedError

    def is_empty(self) -> bool:
        return len(self) == 0


class BatchDataSet:
    def __len__(self) -> int:  # pragma: no cover - interface
        raise NotImplementedError

    def get_batch(self, indices: Sequence[int]) -> List[torch.Tensor]:  # pragma: no cover
        raise NotImplementedError


class TensorDataSet(DataSet, BatchDataSet):
    """A dataset backed by stacked tensors (dim 0 = sample)."""

    def __init__(self, *tensors: torch.Tensor):
        n = tensors[0].shape[0]
        assert all(t.shape[0] == n for t in tensors)
        self.tensors = list(tensors)

    def __len__(self):
        return self.tensors[0].shape[0]

    def get(self, index):
        return [t[index] for t in self.tensors]

    def get_batch(self, indices):
        idx = torch.as_tensor(indices, dtype=torch.long)
        return [t.index_select(0, idx) for t in self.tensors]


class _Batch(list):
    """A batch: list of tensors, with optional names for ``batch["x"]``."""

    def __init__(self, tensors, names=None):
        super().__init__(tensors)
        self.names = names or []

    def __getitem__(self, k):
        if isinstance(k, str):
            return list.__getitem__(self, self.names.index(k))
        return list.__getitem__(self, k)


class DataLoaderBuilder:
    def __init__(self, dataset):
        self._ds = dataset
        self._bs = 32
        self._device = torch.device("cpu")
        self._seed = 0
        self._shuffle = True
        self._sampler: Optional[Sampler] = None
        self._prefetch = 2
        self._vram_max = 0.9
        self._streaming = False
        self._names: List[str] = []
        self._drop_last = False
        self._transform: Optional[Callable] = None
        self._augment = 1

    def batch_size(self, n):
        if n < 1:
            raise ValueError("batch_size must be >= 1")
        self._bs = n
        return self

    def device(self, d):
        self._device = torch.device(d)
        return self

    def seed(self, s):
        self._seed = s
        return self

    def shuffle(self, s=True):
        self._shuffle = s
        return self

    def sampler(self, s: Sampler):
        self._sampler = s
        return self

    def prefetch(self, depth):
        self._prefetch = max(1, depth)
        return self

    def vram_max_usage(self, frac):
        self._vram_max = frac
        return self

    def streaming(self):
        self._streaming = True
        return self

    def names(self, names):
        self._names = list(names)
        return self

    def drop_last(self, d=True):
        self._drop_last = d
        return self

    def transform(self, fn):
        self._transform = fn
        return self

    def augment(self, k):
        self._augment = max(1, k)
        return self

    def build(self) -> "DataLoader":
        return DataLoader(self)


class DataLoader:
    def __init__(self, b: DataLoaderBuilder):
        self.ds = b._ds
        self.bs = b._bs
        self.device_ = b._device
        self.seed_ = b._seed
        self.shuffle_ = b._shuffle
        self.sampler_ = b._sampler
        self.depth = b._prefetch
        self.names_ = b._names
        self.drop_last_ = b._drop_last
        self.transform_ = b._transform
        self.n = len(self.ds)
        self.resident = False
        self._tensors: Optional[List[torch.Tensor]] = None
        if not b._streaming:
            self._try_resident(b._vram_max)

    @classmethod
    def from_dataset(cls, ds) -> DataLoaderBuilder:
        return DataLoaderBuilder(ds)

    from_batch_dataset = from_dataset

    # ------------------------------------------------------------ modes
    def _materialise(self) -> List[torch.Tensor]:
        if isinstance(self.ds, TensorDataSet):
            return [t for t in self.ds.tensors]
        if hasattr(self.ds, "get_batch"):
            return self.ds.get_batch(list(range(self.n)))
        items = [self.ds.get(i) for i in range(self.n)]
        return [torch.stack([it[k] for it in items]) for k in range(len(items[0]))]

    def _try_resident(self, vram_frac: float) -> None:
        tensors = self._materialise()
        nbytes = sum(t.numel() * t.element_size() for t in tensors)
        if self.device_.type == "cuda":
            free, _total = torch.cuda.mem_get_info(self.device_)
            if nbytes > free * vram_frac:
                self._host = tensors
                return
            try:
                self._tensors = [t.to(self.device_) for t in tensors]
            except torch.cuda.OutOfMemoryError:
                torch.cuda.empty_cache()
                self._host = tensors
                return
        else:
            self._tensors = tensors
        self.resident = True

    # ------------------------------------------------------------ API
    def __len__(self):
        return self.num_batches()

    def len(self):
        return self.n

    def _epoch_len(self) -> int:
        if self.sampler_ is not None:
            return len(self.sampler_.indices(0, self.n))
        return self.n

    def num_batches(self) -> int:
        n = self._epoch_len()
        return n // self.bs if self.drop_last_ else math.ceil(n / self.bs)

    def batch_size(self) -> int:
        return self.bs

    def device(self):
        return self.device_

    def is_resident(self) -> bool:
        return self.resident

    def names(self):
        return list(self.names_)

    def prefetch_depth(self) -> int:
        return self.depth

    def set_prefetch_depth(self, d: int) -> None:
        self.depth = max(1, d)

    def _order(self, epoch: int) -> torch.Tensor:
        if self.sampler_ is not None:
            return torch.as_tensor(self.sampler_.indices(epoch, self.n), dtype=torch.long)
        if self.shuffle_:
            g = torch.Generator()
            g.manual_seed(self.seed_ * 1000003 + epoch)
            return torch.randperm(self.n, generator=g)
        return torch.arange(self.n)

    def epoch(self, epoch: int) -> Iterator[_Batch]:
        order = self._order(epoch)
        n = order.numel()
        nb = n // self.bs if self.drop_last_ else math.ceil(n / self.bs)
        if self.resident:
            dev_order = order.to(self._tensors[0].device)
            for i in range(nb):
                idx = dev_order[i * self.bs:(i + 1) * self.bs]
                batch = [t.index_select(0, idx) for t in self._tensors]
                yield self._post(batch)
            return
        from .prefetch import Prefetcher

        host = getattr(self, "_host", None) or self._materialise()
        self._host = host
        pf = Prefetcher(host, order, self.bs, nb, self.device_, self.depth)
        try:
            for batch in pf:
                yield self._post(batch)
        finally:
            pf.close()

    def __iter__(self):
        return self.epoch(0)

    def _post(self, batch):
        if self.transform_ is not None:
            batch = self.transform_(batch)
        return _Batch(batch, self.names_)
