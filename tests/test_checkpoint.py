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


# ------------------------------------------------------------------ reference-format fixture
def _ref_structural_hash():
    """SHA-256 over the fields the reference hashes (flodl/src/graph/checkpoint.rs
    compute_structural_hash), written out field by field for the graph
    Linear(4, 8) -[tag enc]-> GELU -> Linear(8, 2): nodes in topological order
    with their module names and sorted (parameter, shape) lists, the edges, the
    tags with (node index, port index), then the exposed input and output ports.
    Independent of this package's Graph.structural_hash."""
    import hashlib
    h = hashlib.sha256()
    z = b"\0"
    i64 = lambda v: struct.pack("<q", v)
    u64 = lambda v: struct.pack("<Q", v)
    h.update(b"linear_1" + z + b"linear" + z)
    h.update(b"P" + b"bias" + z + i64(8))
    h.update(b"P" + b"weight" + z + i64(8) + i64(4))
    h.update(b"gelu_2" + z + b"gelu" + z)
    h.update(b"linear_3" + z + b"linear" + z)
    h.update(b"P" + b"bias" + z + i64(2))
    h.update(b"P" + b"weight" + z + i64(2) + i64(8))
    h.update(b"EDGES")
    h.update(b"linear_1" + z + b"output" + z + b"gelu_2" + z + b"input" + z)
    h.update(b"gelu_2" + z + b"output" + z + b"linear_3" + z + b"input" + z)
    h.update(b"TAGS" + b"enc" + z + u64(0) + u64(0))
    h.update(b"INPUTS" + b"input" + z + b"linear_1" + z + b"input" + z)
    h.update(b"OUTPUTS" + b"output" + z + b"linear_3" + z + b"output" + z)
    return h.hexdigest()


def _ref_fdl_bytes(hash_hex, entries):
    """A .fdl file assembled by hand from the reference's layout
    (flodl/src/nn/checkpoint.rs save_checkpoint / write_tensor_data):
    MAGIC | u32 version 2 | 32-byte hash | u32 count | entries, each
    u32 name_len | name | u32 ndim | i64 dims | u8 dtype tag | u64 nbytes | raw."""
    out = bytearray(b"FDLC" + struct.pack("<I", 2) + bytes.fromhex(hash_hex) +
                    struct.pack("<I", len(entries)))
    for name, t in entries:
        nb = name.encode()
        out += struct.pack("<I", len(nb)) + nb + struct.pack("<I", t.dim())
        out += b"".join(struct.pack("<q", d) for d in t.shape)
        raw = t.contiguous().numpy().tobytes()
        out += bytes([3]) + struct.pack("<Q", len(raw)) + raw
    return bytes(out)


def test_structural_hash_matches_the_reference_algorithm():
    assert _build(0).structural_hash() == _ref_structural_hash()


def test_loads_a_hand_assembled_reference_checkpoint(tmp_path):
    torch.manual_seed(5)
    want = {"enc/weight": torch.randn(8, 4), "enc/bias": torch.randn(8),
            "linear_3/weight": torch.randn(2, 8), "linear_3/bias": torch.randn(2)}
    order = ["enc/weight", "enc/bias", "linear_3/weight", "linear_3/bias"]
    blob = _ref_fdl_bytes(_ref_structural_hash(), [(k, want[k]) for k in order])
    p = tmp_path / "ref.fdl"
    p.write_bytes(blob)
    g = _build(1)
    rep = load_model(g, str(p))  # validates the structural hash
    assert sorted(rep.loaded) == sorted(order) and not rep.missing and not rep.skipped
    got = dict(g.graph_named_parameters())
    for k in order:
        torch.testing.assert_close(got[k].detach(), want[k])
    # this package writes the same bytes for the same model
    q = tmp_path / "ours.fdl"
    save_model(g, str(q))
    assert q.read_bytes() == blob
    # a different architecture is refused by the hash
    other = FlowBuilder.from_(Linear(4, 8)).tag("enc").through(GELU()).through(Linear(8, 3)).build()
    with pytest.raises(Exception):
        load_model(other, str(p))
