"""HuggingFace families on the sm_100a kernels: each family's masked-LM and
sequence classifier on CUDA (bf16 tensor-core GEMMs, flash attention with the
padding mask) against the same weights in fp32 on the CPU."""
import pytest
import torch

transformers = pytest.importorskip("transformers")
pytestmark = pytest.mark.gpu

from flodl_b200.hf import AutoModelForMaskedLM, AutoModelForSequenceClassification  # noqa: E402

T = transformers
_CFGS = {
    "Bert": lambda: T.BertConfig(vocab_size=512, hidden_size=128, num_hidden_layers=2, num_attention_heads=2,
                                 intermediate_size=256, max_position_embeddings=128),
    "Roberta": lambda: T.RobertaConfig(vocab_size=512, hidden_size=128, num_hidden_layers=2,
                                       num_attention_heads=2, intermediate_size=256,
                                       max_position_embeddings=130),
    "DistilBert": lambda: T.DistilBertConfig(vocab_size=512, dim=128, n_layers=2, n_heads=2, hidden_dim=256,
                                             max_position_embeddings=128),
    "Albert": lambda: T.AlbertConfig(vocab_size=512, embedding_size=64, hidden_size=128, num_hidden_layers=2,
                                     num_attention_heads=2, intermediate_size=256,
                                     max_position_embeddings=128),
    "DebertaV2": lambda: T.DebertaV2Config(vocab_size=512, hidden_size=128, num_hidden_layers=2,
                                           num_attention_heads=2, intermediate_size=256,
                                           max_position_embeddings=128, relative_attention=True,
                                           position_buckets=32, pos_att_type="p2c|c2p",
                                           share_att_key=True, norm_rel_ebd="layer_norm"),
}


@pytest.mark.parametrize("family", list(_CFGS))
@pytest.mark.parametrize("head,auto", [("ForMaskedLM", AutoModelForMaskedLM),
                                       ("ForSequenceClassification", AutoModelForSequenceClassification)])
def test_family_on_cuda_matches_cpu(tmp_path, family, head, auto):
    torch.manual_seed(0)
    hf = getattr(T, family + head)(_CFGS[family]()).eval()
    d = str(tmp_path / "m")
    hf.save_pretrained(d, safe_serialization=True)
    cpu = auto.from_pretrained(d).eval()
    gpu = auto.from_pretrained(d, device="cuda").eval()
    ids = torch.randint(3, 512, (4, 64))
    mask = torch.ones_like(ids)
    mask[1, 40:] = 0
    mask[3, 17:] = 0
    with torch.no_grad():
        ref = cpu(ids, attention_mask=mask).float()
        got = gpu(ids.cuda(), attention_mask=mask.cuda()).float().cpu()
    if ref.dim() == 3:
        ref, got = ref[mask.bool()], got[mask.bool()]
    err = (got - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err < 0.05 * scale + 0.05, (family, head, err, scale)
