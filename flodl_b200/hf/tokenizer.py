"""Tokenizer front end over a HuggingFace ``tokenizer.json``.

Reference: flodl-hf/src/tokenizer.rs (``HfTokenizer`` over the HuggingFace
``tokenizers`` library: model-agnostic, the loaded file carries the
pre-tokenizer and post-processor). ``encode`` pads a batch to its longest
sequence and returns int64 ``[B, S]`` tensors: ``input_ids``,
``attention_mask`` (1 = token, 0 = padding), ``token_type_ids``,
``position_ids`` (``0..S`` per row; RoBERTa-family models derive their own) and
``sequence_ids`` (0 / 1 for the first / second text of a pair, -1 for special
tokens and padding - the signal QA pipelines use to find the context span).

``encode_on_device`` stages the batch in pinned host memory and copies it with
one asynchronous host-to-device copy per tensor on the current stream.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch


@dataclass
class EncodedBatch:
    input_ids: torch.Tensor
    attention_mask: torch.Tensor
    token_type_ids: torch.Tensor
    position_ids: torch.Tensor
    sequence_ids: torch.Tensor

    def to(self, device, non_blocking: bool = True) -> "EncodedBatch":
        f = lambda t: t.to(device, non_blocking=non_blocking)
        return EncodedBatch(f(self.input_ids), f(self.attention_mask), f(self.token_type_ids),
                            f(self.position_ids), f(self.sequence_ids))


class HfTokenizer:
    def __init__(self, inner):
        self.inner = inner
        pad = inner.padding
        self.pad_id = pad["pad_id"] if pad else (inner.token_to_id("[PAD]") or
                                                 inner.token_to_id("<pad>") or 0)
        inner.enable_padding(pad_id=self.pad_id,
                             pad_token=inner.id_to_token(self.pad_id) or "[PAD]")

    @staticmethod
    def from_file(path: str) -> "HfTokenizer":
        from tokenizers import Tokenizer
        return HfTokenizer(Tokenizer.from_file(path))

    @staticmethod
    def from_pretrained(name_or_path: str) -> "HfTokenizer":
        """``tokenizer.json`` of a local model directory or of a Hub repo id
        (through the HuggingFace cache)."""
        import os
        from .auto import resolve_model_dir
        return HfTokenizer.from_file(os.path.join(resolve_model_dir(name_or_path), "tokenizer.json"))

    def save(self, path: str) -> None:
        self.inner.save(path)

    def _batch(self, encs) -> EncodedBatch:
        B = len(encs)
        S = max((len(e.ids) for e in encs), default=0)
        ids = torch.tensor([e.ids for e in encs], dtype=torch.int64).reshape(B, S)
        am = torch.tensor([e.attention_mask for e in encs], dtype=torch.int64).reshape(B, S)
        tt = torch.tensor([e.type_ids for e in encs], dtype=torch.int64).reshape(B, S)
        sq = torch.tensor([[-1 if s is None else s for s in e.sequence_ids] for e in encs],
                          dtype=torch.int64).reshape(B, S)
        pos = torch.arange(S, dtype=torch.int64).expand(B, S).contiguous()
        return EncodedBatch(ids, am, tt, pos, sq)

    def encode(self, texts: Sequence[str]) -> EncodedBatch:
        return self._batch(self.inner.encode_batch(list(texts)))

    def encode_pairs(self, pairs: Sequence[Tuple[str, str]]) -> EncodedBatch:
        return self._batch(self.inner.encode_batch([tuple(p) for p in pairs]))

    def _on_device(self, b: EncodedBatch, device) -> EncodedBatch:
        dev = torch.device(device)
        if dev.type != "cuda":
            return b.to(dev)
        pin = lambda t: t.pin_memory()
        return EncodedBatch(pin(b.input_ids), pin(b.attention_mask), pin(b.token_type_ids),
                            pin(b.position_ids), pin(b.sequence_ids)).to(dev)

    def encode_on_device(self, texts: Sequence[str], device) -> EncodedBatch:
        return self._on_device(self.encode(texts), device)

    def encode_pairs_on_device(self, pairs: Sequence[Tuple[str, str]], device) -> EncodedBatch:
        return self._on_device(self.encode_pairs(pairs), device)

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        return self.inner.decode(list(ids), skip_special_tokens=skip_special_tokens)

    def vocab_size(self) -> int:
        return self.inner.get_vocab_size()


def build_extended_attention_mask(mask: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    """``[B, S]`` 0/1 mask -> additive ``[B, 1, 1, S]`` mask (0 keep, large
    negative drop) for attention implementations that take an additive bias."""
    m = mask[:, None, None, :].to(dtype)
    return (1.0 - m) * torch.finfo(dtype).min
