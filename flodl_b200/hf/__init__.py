"""HuggingFace integration: safetensors IO, BERT/RoBERTa/XLM-R/DistilBERT/ALBERT
loading with task heads, export, and the tokenizer front end."""
from .auto import (AutoModel, AutoModelForMaskedLM, AutoModelForQuestionAnswering,  # noqa: F401
                   AutoModelForSequenceClassification, AutoModelForTokenClassification, export_hf)
from .safetensors_io import load_safetensors, save_safetensors  # noqa: F401
from .tokenizer import EncodedBatch, HfTokenizer, build_extended_attention_mask  # noqa: F401
