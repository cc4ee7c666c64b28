"""Model zoo: the benchmark models of the reference's configs."""
from .bert import (BertConfig, BertForMaskedLM, BertForQuestionAnswering,  # noqa: F401
                   BertForSequenceClassification, BertForTokenClassification, BertModel)
from .transformer_lm import DecoderBlock, TransformerLM  # noqa: F401
from .resnet import BasicBlock, ResNet20  # noqa: F401
from .zoo import ZOO, CharRNN, ModelDef, OLMo  # noqa: F401
from .encoders import (AlbertConfig, AlbertForMaskedLM, AlbertForQuestionAnswering,  # noqa: F401
                       AlbertForSequenceClassification, AlbertForTokenClassification, AlbertModel,
                       DistilBertConfig, DistilBertForMaskedLM, DistilBertForQuestionAnswering,
                       DistilBertForSequenceClassification, DistilBertForTokenClassification,
                       DistilBertModel, RobertaConfig, RobertaForMaskedLM,
                       RobertaForQuestionAnswering, RobertaForSequenceClassification,
                       RobertaForTokenClassification, RobertaModel)
from .deberta import (DebertaV2Config, DebertaV2ForMaskedLM, DebertaV2ForQuestionAnswering,  # noqa: F401
                      DebertaV2ForSequenceClassification, DebertaV2ForTokenClassification,
                      DebertaV2Model)
