"""Model zoo: the benchmark models of the reference's configs."""
from .bert import (BertConfig, BertForMaskedLM, BertForQuestionAnswering,  # noqa: F401
                   BertForSequenceClassification, BertForTokenClassification, BertModel)
from .transformer_lm import DecoderBlock, TransformerLM  # noqa: F401
from .resnet import BasicBlock, ResNet20  # noqa: F401
from .zoo import ZOO, CharRNN, ModelDef, OLMo  # noqa: F401
