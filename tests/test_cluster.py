"""Cluster envelope, builder validation, model signature and test discovery
(reference: cluster_tests.rs, cluster_builder.rs tests, model_sig.rs tests,
testing.rs)."""
import json
import threading

import pytest
import torch

from flodl_b200.parallel.cluster import (ENV_CLUSTER_JSON, ENV_LOCAL_RANK, ENV_TESTING_CLUSTER_JSON,
                                         ClusterBuilder, ClusterError, FullCluster, LocalCluster,
                                         discover_test_cluster, is_reserved_cluster_env_key,
                                         model_sig, module_sig)
from flodl_b200.parallel.rendezvous import RendezvousServer, rendezvous


def _two_hosts():
    return (ClusterBuilder().controller("ctl").port(29511).path("/work").done()
            .host("a").ranks([0, 1]).devices([0, 1]).env("NCCL_DEBUG", "WARN").done()
            .host("b").ranks([2, 3]).all_devices().done()
            .env("FLODL_VERBOSITY", "2").build())


def test_builder_validates_ranks_devices_env():
    fc = _two_hosts()
    assert fc.world_size == 4
    with pytest.raises(ClusterError, match="no duplicates or gaps"):
        (ClusterBuilder().controller("c").done().host("a").ranks([0, 2]).all_devices().done().build())
    with pytest.raises(ClusterError, match="length mismatch"):
        (ClusterBuilder().controller("c").done().host("a").ranks([0, 1]).devices([0]).done().build())
    with pytest.raises(ClusterError, match="reserved"):
        (ClusterBuilder().controller("c").done().host("a").ranks([0]).all_devices()
         .env("CUDA_VISIBLE_DEVICES", "3").done().build())
    with pytest.raises(ClusterError, match="reserved"):
        (ClusterBuilder().controller("c").done().host("a").ranks([0]).all_devices().done()
         .env("FLODL_INTERNAL_ROLE", "x").build())
    with pytest.raises(ClusterError, match="at least one worker"):
        ClusterBuilder().controller("c").done().build()
    ClusterBuilder().controller("c").discovery(True).done().build()  # roster-free window
    with pytest.raises(ClusterError, match="incomplete"):
        ClusterBuilder().controller("c").done().host("a").ranks([0]).done().build()
    with pytest.raises(ClusterError, match="gpu_ram_share"):
        (ClusterBuilder().controller("c").done().host("a").ranks([0]).all_devices().done()
         .gpu_ram_share(-1.0).build())
    assert is_reserved_cluster_env_key("FLODL_INTERNAL_X") and not is_reserved_cluster_env_key("FLODL_VERBOSITY")


def test_envelope_roundtrip_and_my_rank():
    fc = _two_hosts().with_session_salt(bytes(range(16)))
    env = fc.rank_env("b", 1)
    assert env["FLODL_VERBOSITY"] == "2" and "NCCL_DEBUG" not in env  # host a's env only
    lc = LocalCluster.from_env(env)
    assert lc.world_size == 4 and lc.num_workers == 2 and lc.spans_multiple_workers()
    assert lc.worker.ranks == [2, 3] and lc.worker.local_devices == [0, 1]
    assert lc.salt == bytes(range(16)) and lc.worker.path == "/work"
    rank, dev = lc.my_rank(env=env)
    assert rank == 3 and dev == torch.device("cuda", 1)
    rank, dev = lc.my_rank(env={**env, "CUDA_VISIBLE_DEVICES": "1"})
    assert rank == 3 and dev == torch.device("cuda", 0)
    # JSON survives a round trip
    assert LocalCluster.from_value(json.loads(json.dumps(lc.to_json()))) == lc
    # host mismatch is loud
    with pytest.raises(ClusterError, match="does not match"):
        lc.this_worker({"FLODL_HOST_NAME": "elsewhere"})


def test_envelope_parse_errors():
    base = {"controller": {"host": "c", "port": 1}, "world_size": 2, "num_workers": 1,
            "worker": {"host": "a", "ranks": [0, 1], "local_devices": [0, 1]}}
    LocalCluster.from_value(base)
    for bad, msg in (({"world_size": 0}, "world_size"), ({"num_workers": 3}, "exceed"),
                     ({"controller": {"host": "", "port": 1}}, "non-empty"),
                     ({"worker": {"host": "a", "ranks": [0, 5], "local_devices": [0, 1]}}, "out of bounds"),
                     ({"worker": {"host": "a", "ranks": [0, 1], "local_devices": [0]}}, "pair"),
                     ({"salt": "00"}, "salt")):
        with pytest.raises(ClusterError, match=msg):
            LocalCluster.from_value({**base, **bad})


def test_model_sig_binds_name_shape_dtype_and_order():
    w, b = torch.zeros(3, 2), torch.zeros(2)
    base = model_sig([("w", w), ("b", b)], [("rm", torch.zeros(2))])
    assert base == model_sig([("w", w), ("b", b)], [("rm", torch.zeros(2))])
    assert len(base) == 32
    for other in (model_sig([("w2", w), ("b", b)], [("rm", torch.zeros(2))]),
                  model_sig([("w", torch.zeros(2, 3)), ("b", b)], [("rm", torch.zeros(2))]),
                  model_sig([("w", w.double()), ("b", b)], [("rm", torch.zeros(2))]),
                  model_sig([("b", b), ("w", w)], [("rm", torch.zeros(2))]),
                  model_sig([("w", w), ("b", b)], [])):
        assert other != base
    assert module_sig(torch.nn.Linear(4, 3)) == module_sig(torch.nn.Linear(4, 3))
    assert module_sig(torch.nn.Linear(4, 3)) != module_sig(torch.nn.Linear(3, 4))


def test_rendezvous_refuses_model_sig_mismatch():
    key = b"k" * 16
    srv = RendezvousServer(2, key).start()
    errs = []

    def join(i, sig):
        try:
            rendezvous("127.0.0.1", srv.port, key, rank=i, info={"model_sig": sig}, timeout=10)
        except ConnectionError as e:
            errs.append(str(e))

    ts = [threading.Thread(target=join, args=(i, s)) for i, s in ((0, "aa"), (1, "bb"))]
    [t.start() for t in ts]
    [t.join() for t in ts]
    assert len(errs) == 2 and all("model_sig" in e for e in errs)


def test_discover_test_cluster_from_env_and_fallback():
    fc = _two_hosts()
    raw = json.dumps(fc.to_json()).encode().hex()
    got = discover_test_cluster({ENV_TESTING_CLUSTER_JSON: raw})
    assert got.world_size == 4 and [w.host for w in got.workers] == ["a", "b"]
    with pytest.raises(ClusterError, match="hex"):
        discover_test_cluster({ENV_TESTING_CLUSTER_JSON: "not-hex"})
    if not torch.cuda.is_available():
        assert discover_test_cluster({}) is None
