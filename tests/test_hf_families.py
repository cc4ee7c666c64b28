"""HuggingFace family parity on CPU: RoBERTa, XLM-RoBERTa, DistilBERT and
ALBERT (every task head) loaded from `save_pretrained` directories of
randomly initialised transformers models, compared in fp32 with padding;
export round trips back into transformers (reference: flodl-hf parity
scripts and models/*_tests.rs)."""
import pytest
import torch

transformers = pytest.importorskip("transformers")

from flodl_b200.hf import (AutoModel, AutoModelForMaskedLM, AutoModelForQuestionAnswering,  # noqa: E402
                           AutoModelForSequenceClassification, AutoModelForTokenClassification,
                           export_hf)

T = transformers
V = 120


def _cfg(family):
    if family in ("roberta", "xlm-roberta"):
        cls = T.RobertaConfig if family == "roberta" else T.XLMRobertaConfig
        return cls(vocab_size=V, hidden_size=32, num_hidden_layers=2, num_attention_heads=2,
                   intermediate_size=64, max_position_embeddings=40, num_labels=3)
    if family == "distilbert":
        return T.DistilBertConfig(vocab_size=V, dim=32, n_layers=2, n_heads=2, hidden_dim=64,
                                  max_position_embeddings=40, num_labels=3)
    return T.AlbertConfig(vocab_size=V, embedding_size=16, hidden_size=32, num_hidden_layers=3,
                          num_attention_heads=2, intermediate_size=64, max_position_embeddings=40,
                          num_labels=3)


_HF = {"roberta": "Roberta", "xlm-roberta": "XLMRoberta", "distilbert": "DistilBert", "albert": "Albert"}
_HEADS = [("Model", AutoModel), ("ForMaskedLM", AutoModelForMaskedLM),
          ("ForSequenceClassification", AutoModelForSequenceClassification),
          ("ForTokenClassification", AutoModelForTokenClassification),
          ("ForQuestionAnswering", AutoModelForQuestionAnswering)]


def _inputs(family):
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(3, V, (2, 12), generator=g)
    mask = torch.ones_like(ids)
    mask[1, 8:] = 0
    if family in ("roberta", "xlm-roberta"):
        ids[1, 8:] = 1  # RoBERTa pad id: positions skip it
    return ids, mask


def _hf_out(m, ids, mask):
    with torch.no_grad():
        o = m(input_ids=ids, attention_mask=mask)
    if hasattr(o, "start_logits"):
        return o.start_logits, o.end_logits
    return o.logits if hasattr(o, "logits") else o.last_hidden_state


def _ours_out(m, ids, mask):
    with torch.no_grad():
        return m(ids, attention_mask=mask)


def _cmp(a, b, mask, seq_level):
    if isinstance(a, tuple):
        for x, y in zip(a, b):
            torch.testing.assert_close(x[mask.bool()], y[mask.bool()], rtol=2e-4, atol=2e-4)
        return
    if seq_level:
        torch.testing.assert_close(a, b, rtol=2e-4, atol=2e-4)
    else:
        torch.testing.assert_close(a[mask.bool()], b[mask.bool()], rtol=2e-4, atol=2e-4)


@pytest.mark.parametrize("family", ["roberta", "xlm-roberta", "distilbert", "albert"])
@pytest.mark.parametrize("head", [h for h, _ in _HEADS])
def test_family_head_parity_and_export(tmp_path, family, head):
    torch.manual_seed(0)
    hf_cls = getattr(T, _HF[family] + head)
    cfg = _cfg(family)
    if head == "ForQuestionAnswering":
        cfg.num_labels = 2  # start / end
    hf = hf_cls(cfg).eval()
    d = str(tmp_path / "hf")
    hf.save_pretrained(d, safe_serialization=True)
    auto = dict(_HEADS)[head]
    ours = auto.from_pretrained(d).eval()
    assert not ours.load_report, ours.load_report
    ids, mask = _inputs(family)
    ref = _hf_out(hf, ids, mask)
    got = _ours_out(ours, ids, mask)
    seq_level = head == "ForSequenceClassification"
    _cmp(got, ref, mask, seq_level)
    out = str(tmp_path / "export")
    export_hf(ours, out)
    hf2 = hf_cls.from_pretrained(out).eval()
    _cmp(_hf_out(hf2, ids, mask), ref, mask, seq_level)


def test_deberta_v2_is_refused_clearly(tmp_path):
    cfg = T.DebertaV2Config(vocab_size=V, hidden_size=32, num_hidden_layers=1, num_attention_heads=2,
                            intermediate_size=64)
    d = str(tmp_path / "deb")
    T.DebertaV2Model(cfg).save_pretrained(d, safe_serialization=True)
    with pytest.raises(NotImplementedError, match="deberta-v2"):
        AutoModel.from_pretrained(d)
