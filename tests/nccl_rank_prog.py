"""Child program for tests/test_runtime_utils.py: one gloo rank of the
communicator layer."""
import json
import sys

import torch

from flodl_b200.parallel.nccl import NcclRankComm, NcclUniqueId, ReduceOp

rank, world, raw = int(sys.argv[1]), int(sys.argv[2]), bytes.fromhex(sys.argv[3])
c = NcclRankComm.init_rank(rank, world, NcclUniqueId(raw), "cpu", timeout_s=60)
out = {}
t = torch.full((4,), float(rank + 1))
c.all_reduce([t], ReduceOp.Sum)
out["sum"] = t.tolist()
t = torch.full((4,), float(rank + 1))
c.all_reduce_premul_sum([t], 0.5 * (rank + 1))
out["premul"] = t.tolist()
b = torch.full((2,), float(rank))
c.broadcast([b], root=world - 1)
out["bcast"] = b.tolist()
out["per_rank"] = c.all_reduce_per_rank_f64(10.0 * rank)
sub = c.split(rank % 2)
s = torch.full((1,), float(rank))
sub.all_reduce([s])
out["split"] = [sub.rank, sub.world, s.item()]
c.abort_handle.abort()
c.abort_handle.abort()  # idempotent
c.close()
print(json.dumps(out))
