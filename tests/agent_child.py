"""Rank child for tests/test_agent.py: reads its envelope and records its rank."""
import json
import os
import sys

from flodl_b200.parallel.cluster import LocalCluster

lc = LocalCluster.from_env()
rank, _dev = lc.my_rank()
out = sys.argv[1]
with open(os.path.join(out, f"rank{rank}.json"), "w") as f:
    json.dump({"rank": rank, "world": lc.world_size, "host": lc.worker.host,
               "local": int(os.environ["FLODL_INTERNAL_LOCAL_RANK"])}, f)
sys.exit(int(os.environ.get("FAIL_RANK", "-1") == str(rank)) * 7)
