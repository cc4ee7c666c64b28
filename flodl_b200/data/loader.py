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

Streaming reads fall through the staging cascade of
:mod:`flodl_b200.data.staging`: a device sample pool (``vram_pool``), a RAM
sample cache (``sample_cache``, sized by ``ram_max_usage``), an optional
local disk stage (``disk_stage``), then the dataset. Without an explicit
``prefetch`` depth, the depth fills ``vram_max_usage`` of the device minus
``step_reserve`` with batches. ``augment(k)`` schedules every sample ``k``
times per epoch (variation comes from ``transform``).
"""
from __future__ import annotations

import math
from typing import Callable, Iterator, List, Optional, Sequence

import torch

from .sampler import RandomSampler, Sampler, SequentialSampler

HOST_RESIDENT_FRAC = 0.5  # a CPU-target dataset stays resident within this share of RAM


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
        self._prefetch_set = False
        self._ram_max = 0.5
        self._gpu_ram_share: Optional[float] = None
        self._sample_cache = True
        self._disk_gb = 0.0
        self._disk_dir: Optional[str] = None
        self._vram_pool = True
        self._step_reserve: Optional[int] = None

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
        self._prefetch_set = True
        return self

    def ram_max_usage(self, frac):
        """Host-RAM share for the sample cache (clamped to [0, 0.9]; 0 = off)."""
        self._ram_max = min(max(frac, 0.0), 0.9)
        return self

    def gpu_ram_share(self, share):
        """Unified-memory parts: the GPU's share of MemTotal, kept out of host budgets."""
        if not share >= 0:
            raise ValueError("gpu_ram_share must be >= 0")
        self._gpu_ram_share = share
        return self

    def sample_cache(self, on=True):
        self._sample_cache = on
        return self

    def disk_stage(self, gb):
        """Local-disk overflow tier below the sample cache, in GB (0 = off)."""
        self._disk_gb = max(0.0, gb)
        return self

    def disk_stage_dir(self, path):
        self._disk_dir = path
        return self

    def vram_pool(self, on=True):
        self._vram_pool = on
        return self

    def step_reserve(self, nbytes):
        """Device bytes to keep free for the training step when sizing prefetch."""
        self._step_reserve = int(nbytes)
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
        if self._augment > 1 and self._sampler is not None:
            raise ValueError("augment(k > 1) composes with the built-in samplers only")
        if self._disk_gb > 0 and (not self._sample_cache or
                                  (isinstance(self._ds, BatchDataSet) and not isinstance(self._ds, DataSet))):
            raise ValueError("disk_stage needs the sample layer: a per-sample DataSet with sample_cache on")
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
        self.augment_ = b._augment
        self.vram_max_ = b._vram_max
        self.auto_depth = not b._prefetch_set
        self.step_reserve_ = b._step_reserve
        self.n = len(self.ds)
        self.resident = False
        self._tensors: Optional[List[torch.Tensor]] = None
        self._b = b
        self.cache = self.disk = self.pool = None
        if not b._streaming:
            self._try_resident(b._vram_max)
        if not self.resident:
            self._setup_streaming()

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

    def _estimate_bytes(self) -> int:
        if isinstance(self.ds, TensorDataSet):
            return sum(t.numel() * t.element_size() for t in self.ds.tensors)
        if self.n == 0:
            return 0
        one = self.ds.get_batch([0]) if hasattr(self.ds, "get_batch") else self.ds.get(0)
        per = sum(t.numel() * t.element_size() for t in one)
        return per * self.n

    def _try_resident(self, vram_frac: float) -> None:
        from . import staging
        est = self._estimate_bytes()
        if self.device_.type == "cuda":
            free, _total = torch.cuda.mem_get_info(self.device_)
            if est > free * vram_frac:
                return  # streaming: nothing materialised
        elif est > staging.host_budget(HOST_RESIDENT_FRAC, staging.host_available_bytes()):
            return
        tensors = self._materialise()
        if self.device_.type == "cuda":
            try:
                self._tensors = [t.to(self.device_) for t in tensors]
            except torch.cuda.OutOfMemoryError:
                torch.cuda.empty_cache()
                if not self._per_sample():
                    self._host = tensors
                return
        else:
            self._tensors = tensors
        self.resident = True

    def _per_sample(self) -> bool:
        return not isinstance(self.ds, TensorDataSet) and not hasattr(self.ds, "get_batch")

    def _setup_streaming(self) -> None:
        from . import staging
        b = self._b
        if self._per_sample() and b._sample_cache and b._ram_max > 0:
            avail = staging.host_available_bytes(b._gpu_ram_share)
            self.cache = staging.SampleCache(staging.host_budget(b._ram_max, avail))
        if self._per_sample() and b._disk_gb > 0:
            self.disk = staging.DiskStage(int(b._disk_gb * (1 << 30)), b._disk_dir)
        self._use_pool = b._vram_pool and self.device_.type == "cuda"

    def _read_sample(self, i: int) -> List[torch.Tensor]:
        if self.cache is not None:
            v = self.cache.get(i)
            if v is not None:
                return v
        if self.disk is not None:
            v = self.disk.get(i)
            if v is not None:
                return v
        v = self.ds.get(i)
        if self.cache is None or not self.cache.admit(i, v):
            if self.disk is not None:
                self.disk.admit(i, v)
        return v

    def fetch(self, idx: torch.Tensor) -> List[torch.Tensor]:
        """Host rows of samples ``idx`` through the staging cascade."""
        if self._tensors is not None:
            return [t.index_select(0, idx.to(t.device)) for t in self._tensors]
        host = getattr(self, "_host", None)
        if host is not None:
            return [t.index_select(0, idx) for t in host]
        if isinstance(self.ds, TensorDataSet):
            return [t.index_select(0, idx) for t in self.ds.tensors]
        if hasattr(self.ds, "get_batch"):
            return self.ds.get_batch(idx.tolist())
        items = [self._read_sample(int(i)) for i in idx]
        return [torch.stack([it[k] for it in items]) for k in range(len(items[0]))]

    def _make_pool(self, sample_rows: List[torch.Tensor]):
        from . import staging
        if self.pool is not None or not self._use_pool:
            return self.pool
        row_bytes = sum(r[0].numel() * r.element_size() for r in sample_rows)
        free, total = torch.cuda.mem_get_info(self.device_)
        used = total - free
        reserve = self.step_reserve_ or 0
        room = min(max(self.vram_max_, 0.5), 0.99) * total - used - reserve
        room -= self.depth * row_bytes * self.bs  # the prefetch ring comes first
        cap = int(max(0, room // 2) // max(row_bytes, 1))  # half the leftover, the step grows
        cap = min(cap, self.n)
        if cap > 0:
            self.pool = staging.VramPool(cap, [tuple(r.shape[1:]) for r in sample_rows],
                                         [r.dtype for r in sample_rows], self.device_)
        return self.pool

    def _auto_depth(self, sample_rows: List[torch.Tensor]) -> None:
        from . import staging
        if not self.auto_depth or self.device_.type != "cuda":
            return
        batch_bytes = sum(r[0].numel() * r.element_size() for r in sample_rows) * self.bs
        free, total = torch.cuda.mem_get_info(self.device_)
        reserve = self.step_reserve_ if self.step_reserve_ is not None else 0
        d = staging.prefetch_depth(self.vram_max_, total, total - free, batch_bytes, reserve)
        self.depth = d if self.step_reserve_ is not None else max(2, d // 3)

    def staging_stats(self) -> dict:
        out = {}
        if self.cache is not None:
            out["cache"] = {"held": len(self.cache), "hits": self.cache.hits, "misses": self.cache.misses}
        if self.disk is not None:
            out["disk"] = {"held": len(self.disk.index), "hits": self.disk.hits}
        if self.pool is not None:
            out["pool"] = {"held": self.pool.used, "capacity": self.pool.capacity,
                           "hits": self.pool.hits, "misses": self.pool.misses}
        return out

    def close(self) -> None:
        if self.disk is not None:
            self.disk.close()
            self.disk = None

    # ------------------------------------------------------------ API
    def __len__(self):
        return self.num_batches()

    def len(self):
        return self.n

    def _epoch_len(self) -> int:
        if self.sampler_ is not None:
            return len(self.sampler_.indices(0, self.n))
        return self.n * self.augment_

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
        n = self.n * self.augment_
        if self.shuffle_:
            g = torch.Generator()
            g.manual_seed(self.seed_ * 1000003 + epoch)
            return torch.randperm(n, generator=g) % self.n
        return torch.arange(n) % self.n

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

        first = self.fetch(order[:1])
        self._auto_depth(first)
        pool = self._make_pool(first) if self.device_.type == "cuda" else None
        pf = Prefetcher(self.fetch, order, self.bs, nb, self.device_, self.depth, pool)
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
