"""`.fdl` checkpoint format (reference: flodl/src/nn/checkpoint.rs, checkpoint_tests.rs)."""
import gzip
import struct

import pytest
import torch

from flodl_b200.graph import FlowBuilder
from flodl_b200.nn import (GELU, Linear, checkpoint_keys, checkpoint_version, load_checkpoint,
                           load_model, migrate_checkpoint, read_checkpoint, save_checkpoint,
                           save_model)


def _build(seed=0):
    torch.manual_seed(seed)
    return FlowBuilder.from_(Linear(4, 8)).tag("enc").through(GELU()).through(Linear(8, 2)).build()


def test_byte_layout(tmp_path):
    p = str(tmp_path / "m.fdl")
    t = torch.arange(6, dtype=torch.float32).reshape(2, 3)
    save_checkpoint(p, [("a/weight", t)], [], None)
    raw = open(p, "rb").read()
    assert raw[:4] == b"FDLC"
    assert struct.unpack("<I", raw[4:8])[0] == 2
    assert raw[8:40] == b"\0" * 32
    assert struct.unpack("<I", raw[40:44])[0] == 1
    off = 44
    (nl,) = struct.unpack("<I", raw[off:off + 4]); off += 4
    assert raw[off:off + nl] == b"a/weight"; off += nl
    (nd,) = struct.unpack("<I", raw[off:off + 4]); off += 4
    assert nd == 2 and struct.unpack("<2q", raw[off:off + 16]) == (2, 3); off += 16
    assert raw[off] == 3; off += 1  # f32 tag
    (nb,) = struct.unpack("<Q", raw[off:off + 8]); off += 8
    assert nb == 24 and torch.frombuffer(bytearray(raw[off:off + nb]), dtype=torch.float32).tolist() == list(range(6))
    assert off + nb == len(raw)


@pytest.mark.parametrize("suffix", [".fdl", ".fdl.gz"])
def test_roundtrip_with_hash(tmp_path, suffix):
    g = _build(0)
    p = str(tmp_path / ("m" + suffix))
    save_model(g, p)
    if suffix.endswith(".gz"):
        assert gzip.open(p).read(4) == b"FDLC"
    g2 = _build(1)
    rep = load_model(g2, p)
    assert sorted(rep.loaded) == sorted(n for n, _ in g.graph_named_parameters())
    assert not rep.missing and not rep.skipped
    x = torch.randn(3, 4)
    torch.testing.assert_close(g(x), g2(x))
    assert checkpoint_version(p) == 2
    assert checkpoint_keys(p)[0] == "enc/weight"


def test_hash_mismatch_and_shape_mismatch(tmp_path):
    g = _build(0)
    p = str(tmp_path / "m.fdl")
    save_model(g, p)
    other = FlowBuilder.from_(Linear(4, 9)).tag("enc").through(GELU()).through(Linear(9, 2)).build()
    with pytest.raises(ValueError, match="architecture mismatch"):
        load_model(other, p)
    with pytest.raises(ValueError, match="shape mismatch"):
        load_checkpoint(p, other.graph_named_parameters(), [], None)


def test_report_missing_skipped_and_dtypes(tmp_path):
    p = str(tmp_path / "m.fdl")
    ents = [("x", torch.ones(2, dtype=torch.bfloat16)), ("y", torch.arange(3, dtype=torch.int64)),
            ("z", torch.zeros(1, dtype=torch.float64))]
    save_checkpoint(p, ents)
    ver, h, back = read_checkpoint(p)
    assert [n for n, _ in back] == ["x", "y", "z"]
    assert back[0][1].dtype == torch.bfloat16 and back[1][1].dtype == torch.int64
    tgt = torch.zeros(2)
    rep = load_checkpoint(p, [("x", tgt), ("w", torch.zeros(1))])
    assert rep.loaded == ["x"] and rep.missing == ["w"] and sorted(rep.skipped) == ["y", "z"]
    assert tgt.tolist() == [1.0, 1.0]


def test_atomic_write_leaves_no_tmp(tmp_path):
    p = tmp_path / "m.fdl"
    save_checkpoint(str(p), [("a", torch.ones(1))])
    assert not (tmp_path / "m.fdl.tmp").exists()


def test_migrate_renames(tmp_path):
    src, dst = str(tmp_path / "a.fdl"), str(tmp_path / "b.fdl")
    save_checkpoint(src, [("old/w", torch.ones(2))])
    rep = migrate_checkpoint(src, dst, {"old/w": "new/w"})
    assert rep.renamed == [("old/w", "new/w")]
    assert checkpoint_keys(dst) == ["new/w"]
