"""Rank program for the launcher tests: rendezvous, gloo all-reduce, report.

FAIL_RANK / FAIL_ATTEMPT make one rank exit with an error on one attempt."""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from flodl_b200.parallel.launcher import ENV_ATTEMPT, init_rank  # noqa: E402

attempt = int(os.environ.get(ENV_ATTEMPT, "0"))
if (os.environ.get("FAIL_RANK") == os.environ.get("LOCAL_RANK")
        and int(os.environ.get("FAIL_ATTEMPT", "-1")) == attempt):
    sys.exit(3)
info = init_rank(backend="gloo", timeout_s=60)
t = torch.tensor([float(info.rank + 1)])
dist.all_reduce(t)
out = os.environ["OUT_DIR"]
with open(os.path.join(out, f"rank{info.rank}_attempt{attempt}.json"), "w") as f:
    json.dump({"rank": info.rank, "world": info.world, "sum": t.item()}, f)
dist.destroy_process_group()
