"""HuggingFace integration: safetensors IO, BERT-family loading, export."""
from .auto import (AutoModel, AutoModelForMaskedLM, AutoModelForQuestionAnswering,  # noqa: F401
                   AutoModelForSequenceClassification, AutoModelForTokenClassification, export_hf)
from .safetensors_io import load_safetensors, save_safetensors  # noqa: F401
