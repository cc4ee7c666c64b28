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


def _wordpiece_tokenizer(path):
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers import Tokenizer, models, normalizers, pre_tokenizers, processors
    vocab = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]", "hello", "world", "the", "cat", "sat",
             "on", "mat", "##s", "what", "where", "is", "?", "."]
    tok = Tokenizer(models.WordPiece({w: i for i, w in enumerate(vocab)}, unk_token="[UNK]"))
    tok.add_special_tokens(["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"])
    tok.normalizer = normalizers.BertNormalizer(lowercase=True)
    tok.pre_tokenizer = pre_tokenizers.BertPreTokenizer()
    tok.post_processor = processors.TemplateProcessing(
        single="[CLS] $A [SEP]", pair="[CLS] $A [SEP] $B:1 [SEP]:1",
        special_tokens=[("[CLS]", 2), ("[SEP]", 3)])
    tok.save(path)


def test_tokenizer_batch_pairs_and_masks(tmp_path):
    from flodl_b200.hf.tokenizer import HfTokenizer, build_extended_attention_mask
    p = str(tmp_path / "tokenizer.json")
    _wordpiece_tokenizer(p)
    tok = HfTokenizer.from_file(p)
    b = tok.encode(["Hello world", "the cats sat on the mat."])
    assert b.input_ids.shape == (2, 10) and b.input_ids.dtype == torch.int64
    assert b.input_ids[0].tolist()[:4] == [2, 5, 6, 3] and b.attention_mask[0].tolist() == [1] * 4 + [0] * 6
    assert b.input_ids[1].tolist()[2:4] == [8, 12]  # "cats" -> cat ##s
    assert b.sequence_ids[0].tolist()[:4] == [-1, 0, 0, -1] and b.position_ids[1, -1] == 9
    pr = tok.encode_pairs([("what is the cat", "the cat sat")])
    assert pr.token_type_ids[0].tolist() == [0] * 6 + [1] * 4
    assert pr.sequence_ids[0].tolist() == [-1, 0, 0, 0, 0, -1, 1, 1, 1, -1]
    assert tok.decode(pr.input_ids[0].tolist()) == "what is the cat the cat sat"
    ext = build_extended_attention_mask(b.attention_mask)
    assert ext.shape == (2, 1, 1, 10) and ext[0, 0, 0, 0] == 0 and ext[0, 0, 0, 9] < -1e30
    on = tok.encode_on_device(["hello"], "cpu")
    assert on.input_ids.tolist() == [[2, 5, 3]]


def test_hub_repo_id_resolves_from_cache_offline(tmp_path, monkeypatch):
    transformers = pytest.importorskip("transformers")
    pytest.importorskip("huggingface_hub")
    cfg = transformers.BertConfig(vocab_size=64, hidden_size=32, num_hidden_layers=1, num_attention_heads=2,
                                  intermediate_size=64, max_position_embeddings=32)
    snap = tmp_path / "hub" / "models--acme--tiny-bert" / "snapshots" / "abc123"
    snap.mkdir(parents=True)
    transformers.BertForMaskedLM(cfg).save_pretrained(str(snap), safe_serialization=True)
    refs = tmp_path / "hub" / "models--acme--tiny-bert" / "refs"
    refs.mkdir()
    (refs / "main").write_text("abc123")
    monkeypatch.setenv("HF_HUB_CACHE", str(tmp_path / "hub"))
    monkeypatch.setenv("HF_HUB_OFFLINE", "1")

    import huggingface_hub.constants as hc
    monkeypatch.setattr(hc, "HF_HUB_CACHE", str(tmp_path / "hub"))
    monkeypatch.setattr(hc, "HF_HUB_OFFLINE", True)
    m = AutoModelForMaskedLM.from_pretrained("acme/tiny-bert")
    assert m.config.hidden_size == 32
    with pytest.raises(FileNotFoundError, match="acme/missing"):
        AutoModelForMaskedLM.from_pretrained("acme/missing")
