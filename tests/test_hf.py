"""safetensors IO and HF BERT parity (reference: flodl-hf tests, parity scripts)."""
import os

import pytest
import torch

from flodl_b200.hf import AutoModelForMaskedLM, export_hf, load_safetensors, save_safetensors
from flodl_b200.models import BertConfig, BertForMaskedLM


def test_safetensors_roundtrip(tmp_path):
    p = str(tmp_path / "m.safetensors")
    t = {"a": torch.randn(3, 4), "b": torch.arange(5, dtype=torch.int64), "c": torch.randn(2).bfloat16()}
    save_safetensors(p, t, {"format": "pt"})
    back = load_safetensors(p)
    for k in t:
        assert torch.equal(back[k], t[k])


def test_matches_hf_transformers_bert(tmp_path):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.BertConfig(vocab_size=200, hidden_size=64, num_hidden_layers=2,
                                  num_attention_heads=2, intermediate_size=128,
                                  max_position_embeddings=64)
    torch.manual_seed(0)
    hf = transformers.BertForMaskedLM(cfg).eval()
    d = str(tmp_path / "hfbert")
    hf.save_pretrained(d, safe_serialization=True)
    ours = AutoModelForMaskedLM.from_pretrained(d).eval()
    ids = torch.randint(0, 200, (2, 10))
    mask = torch.ones_like(ids)
    mask[1, 7:] = 0
    with torch.no_grad():
        ref = hf(input_ids=ids, attention_mask=mask).logits
        got = ours(ids, attention_mask=mask)
    valid = mask.bool()
    torch.testing.assert_close(got[valid], ref[valid], rtol=1e-4, atol=1e-4)
    # export round trip
    out = str(tmp_path / "export")
    export_hf(ours, out)
    hf2 = transformers.BertForMaskedLM.from_pretrained(out).eval()
    with torch.no_grad():
        ref2 = hf2(input_ids=ids, attention_mask=mask).logits
    torch.testing.assert_close(ref2[valid], ref[valid], rtol=1e-4, atol=1e-4)
