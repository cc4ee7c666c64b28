"""DataLoader behaviour (reference: flodl/src/data/loader_tests.rs)."""
import torch

from flodl_b200.data import (DataLoader, DataSet, DistributedSampler, TensorDataSet,
                             synthetic_tokens)


class Squares(DataSet):
    def __len__(self):
        return 10

    def get(self, i):
        return [torch.tensor([float(i)]), torch.tensor(i * i)]


def test_resident_epoch_covers_all_and_is_seeded():
    dl = DataLoader.from_dataset(Squares()).batch_size(4).seed(3).build()
    assert dl.is_resident() and dl.num_batches() == 3
    seen = torch.cat([b[0].reshape(-1) for b in dl.epoch(0)]).tolist()
    assert sorted(seen) == [float(i) for i in range(10)]
    again = torch.cat([b[0].reshape(-1) for b in dl.epoch(0)]).tolist()
    other = torch.cat([b[0].reshape(-1) for b in dl.epoch(1)]).tolist()
    assert seen == again and seen != other


def test_streaming_matches_resident_and_drop_last():
    ds = TensorDataSet(torch.arange(20).float().unsqueeze(1), torch.arange(20))
    a = DataLoader.from_dataset(ds).batch_size(6).seed(1).drop_last().build()
    b = DataLoader.from_dataset(ds).batch_size(6).seed(1).drop_last().streaming().build()
    assert not b.is_resident() and a.num_batches() == 3
    ra = [x[1].tolist() for x in a.epoch(2)]
    rb = [x[1].tolist() for x in b.epoch(2)]
    assert ra == rb


def test_names_and_distributed_sampler():
    ds = synthetic_tokens(16, 8, 50)
    dl = DataLoader.from_dataset(ds).batch_size(4).names(["ids", "tgt"]).shuffle(False).build()
    b = next(iter(dl))
    assert b["ids"].shape == (4, 8)
    s0 = DistributedSampler(0, 2, seed=5).indices(0, 10)
    s1 = DistributedSampler(1, 2, seed=5).indices(0, 10)
    assert len(s0) == len(s1) == 5 and sorted(s0 + s1) == list(range(10))


class Counting(DataSet):
    """Per-sample dataset that counts source reads (a slow source stand-in)."""

    def __init__(self, n=40):
        self.n, self.reads = n, 0

    def __len__(self):
        return self.n

    def get(self, i):
        self.reads += 1
        return [torch.full((3,), float(i)), torch.tensor(i)]


def _epoch_ids(dl, e):
    return [int(v) for b in dl.epoch(e) for v in b[1]]


def test_streaming_sample_cache_serves_later_epochs_from_ram():
    ds = Counting()
    dl = DataLoader.from_dataset(ds).batch_size(8).streaming().build()
    assert sorted(_epoch_ids(dl, 0)) == list(range(40))
    assert ds.reads == 40  # the sizing probe's read is cached too
    assert sorted(_epoch_ids(dl, 1)) == list(range(40))
    assert ds.reads == 40 and dl.staging_stats()["cache"]["held"] == 40


def test_disk_stage_takes_what_ram_declines(tmp_path):
    ds = Counting()
    b = DataLoader.from_dataset(ds).batch_size(8).streaming().ram_max_usage(0.0).disk_stage(0.001)
    dl = b.disk_stage_dir(str(tmp_path)).build()
    assert dl.cache is None and dl.disk is not None
    first = _epoch_ids(dl, 0)
    reads = ds.reads
    second = _epoch_ids(dl, 1)
    assert sorted(second) == list(range(40)) and ds.reads == reads
    assert dl.staging_stats()["disk"]["hits"] >= 40
    # rows read back from the pack file equal the source rows
    for batch in dl.epoch(2):
        assert torch.equal(batch[0][:, 0], batch[1].float())
    path = dl.disk.path
    dl.close()
    import os
    assert not os.path.exists(path)


def test_augment_schedules_k_views_and_rejects_custom_sampler():
    ds = TensorDataSet(torch.arange(10).float().unsqueeze(1), torch.arange(10))
    dl = DataLoader.from_dataset(ds).batch_size(5).augment(3).build()
    ids = _epoch_ids(dl, 0)
    assert len(ids) == 30 and sorted(ids) == sorted(list(range(10)) * 3) and dl.num_batches() == 6
    import pytest
    with pytest.raises(ValueError, match="augment"):
        DataLoader.from_dataset(ds).augment(2).sampler(DistributedSampler(0, 2)).build()


def test_budget_law_and_prefetch_depth():
    from flodl_b200.data import staging
    assert staging.host_budget(0.5, 100, 0) == 50
    assert staging.host_budget(2.0, 100, 0) == 90       # hard 0.9 ceiling
    assert staging.host_budget(0.5, 60, 40) == 50       # held bytes added back: anchored
    info = {"MemTotal": 1000, "MemAvailable": 800}
    assert staging.host_available_bytes(0.5, info) == 300  # APU share of the same DRAM removed
    assert staging.prefetch_depth(0.9, 1000, 100, 100) == 8
    assert staging.prefetch_depth(0.9, 1000, 890, 100) == 2
    assert staging.prefetch_depth(0.9, 10 ** 9, 0, 1, max_depth=16) == 16


def test_resolve_cached_prefers_source_then_acquires_once(tmp_path):
    from flodl_b200.data.staging import resolve_cached
    src, cache = tmp_path / "src", tmp_path / "cache"
    (src / "ds").mkdir(parents=True)
    calls = []

    def fetch(dst):
        calls.append(dst)
        with open(dst, "w") as f:
            f.write("data")

    p = resolve_cached(str(src), "ds", "a.bin", lambda p: True, fetch, str(cache))
    assert p == str(cache / "ds" / "a.bin") and len(calls) == 1
    assert resolve_cached(str(src), "ds", "a.bin", lambda p: True, fetch, str(cache)) == p and len(calls) == 1
    (src / "ds" / "b.bin").write_text("x")
    assert resolve_cached(str(src), "ds", "b.bin", lambda p: True, fetch, str(cache)) == str(src / "ds" / "b.bin")


def test_fixed_stride_records_and_cifar_mnist_readers(tmp_path):
    import struct

    import numpy as np

    from flodl_b200.data.datasets import cifar10, mnist
    from flodl_b200.data.records import FixedStrideRecords, cifar10_records, mnist_records
    rng = np.random.default_rng(0)
    for name in [f"data_batch_{i}.bin" for i in range(1, 6)]:
        recs = np.concatenate([rng.integers(0, 10, (7, 1)), rng.integers(0, 256, (7, 3072))], 1)
        recs.astype(np.uint8).tofile(str(tmp_path / name))
    full, streamed = cifar10(str(tmp_path)), cifar10_records(str(tmp_path))
    assert len(streamed) == 35
    for i in (0, 6, 7, 34):
        x, y = streamed.get(i)
        torch.testing.assert_close(x, full.tensors[0][i])
        assert int(y) == int(full.tensors[1][i])
    imgs = rng.integers(0, 256, (5, 28, 28)).astype(np.uint8)
    labs = rng.integers(0, 10, 5).astype(np.uint8)
    (tmp_path / "train-images-idx3-ubyte").write_bytes(struct.pack(">IIII", 0x803, 5, 28, 28) + imgs.tobytes())
    (tmp_path / "train-labels-idx1-ubyte").write_bytes(struct.pack(">II", 0x801, 5) + labs.tobytes())
    m, ms = mnist(str(tmp_path)), mnist_records(str(tmp_path))
    for i in range(5):
        x, y = ms.get(i)
        torch.testing.assert_close(x, m.tensors[0][i])
        assert int(y) == int(m.tensors[1][i])
    import pytest
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"x" * 10)
    with pytest.raises(ValueError, match="whole number"):
        FixedStrideRecords(str(bad), 3)
    dl = DataLoader.from_dataset(streamed).batch_size(8).streaming().build()
    assert sum(b[0].shape[0] for b in dl.epoch(0)) == 35
