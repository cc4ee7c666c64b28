"""Model zoo: the benchmark models of the reference's configs."""
from .transformer_lm import DecoderBlock, TransformerLM  # noqa: F401
