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
