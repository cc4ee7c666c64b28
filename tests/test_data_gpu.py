"""Streaming loader on CUDA: device sample pool and VRAM-sized prefetch."""
import pytest
import torch

from flodl_b200.data import DataLoader, DataSet

pytestmark = pytest.mark.gpu


class Rows(DataSet):
    def __len__(self):
        return 96

    def get(self, i):
        return [torch.full((16,), float(i)), torch.tensor(i)]


def test_vram_pool_serves_second_epoch_on_device():
    dl = DataLoader.from_dataset(Rows()).batch_size(16).device("cuda").streaming().build()
    for e in range(2):
        seen = []
        for x, y in dl.epoch(e):
            assert x.is_cuda and torch.equal(x[:, 0].long(), y)
            seen += y.tolist()
        assert sorted(seen) == list(range(96))
    st = dl.staging_stats()
    assert st["pool"]["held"] == 96 and st["pool"]["hits"] >= 96
    assert dl.prefetch_depth() >= 2
