"""Tokenizer wrapper (reference ``mamformer/tokenizer.py``).

Wraps a HuggingFace tokenizer, or falls back to a character-level tokenizer (vocab 256,
pad 0, bos 1, eos 2; characters outside the vocab map to a space).  Thinking control tokens
have fixed ids 3..7.
"""

from __future__ import annotations

import logging
import warnings
from typing import Dict, List, Optional, Union


class MamformerTokenizer:
    THINK_START_ID: int = 3
    THINK_END_ID: int = 4
    ANSWER_START_ID: int = 5
    ANSWER_END_ID: int = 6
    SUMMARY_START_ID: int = 7
    THINKING_TOKEN_IDS = {3, 4, 5, 6, 7}
    THINKING_TOKEN_NAMES: Dict[int, str] = {3: "<|think_start|>", 4: "<|think_end|>",
                                            5: "<|answer_start|>", 6: "<|answer_end|>",
                                            7: "<|summary_start|>"}

    def __init__(self, tokenizer=None, bos_token: str = "<s>", eos_token: str = "</s>",
                 pad_token: str = "<pad>") -> None:
        self._tokenizer = tokenizer
        self.think_start_token_id = self.THINK_START_ID
        self.think_end_token_id = self.THINK_END_ID
        self.answer_start_token_id = self.ANSWER_START_ID
        self.answer_end_token_id = self.ANSWER_END_ID
        self.summary_start_token_id = self.SUMMARY_START_ID
        self._bos, self._eos, self._pad = bos_token, eos_token, pad_token
        if tokenizer is not None:
            self.bos_token_id = tokenizer.bos_token_id or 0
            self.eos_token_id = tokenizer.eos_token_id or 1
            self.pad_token_id = tokenizer.pad_token_id or 0
            self.vocab_size = max(tokenizer.vocab_size, self.answer_end_token_id + 1)
        else:
            self.bos_token_id, self.eos_token_id, self.pad_token_id = 1, 2, 0
            self.vocab_size = max(256, self.answer_end_token_id + 1)

    # -- char-level fallback --------------------------------------------------------------
    def _encode_one(self, text: str, **kw) -> List[int]:
        if self._tokenizer is not None:
            return list(self._tokenizer.encode(text, **kw))
        out, warned = [], False
        for ch in text:
            c = ord(ch)
            if 0 < c < self.vocab_size:
                out.append(c)
            else:
                if not warned:
                    warnings.warn(f"Character {ch!r} exceeds vocab_size={self.vocab_size}; mapped to space.")
                    warned = True
                out.append(32)
        return out

    def _decode_ids(self, ids: List[int], **kw) -> str:
        if self._tokenizer is not None:
            return self._tokenizer.decode(ids, **kw)
        out = []
        for t in ids:
            if 0 < t < self.vocab_size:
                out.append(chr(t))
            elif t == self.eos_token_id:
                break
            else:
                out.append("�")
        return "".join(out)

    def encode(self, text: Union[str, List[str]], add_bos: bool = True, add_eos: bool = False,
               max_length: Optional[int] = None, truncation: bool = False, padding: bool = False,
               **kw) -> Union[List[int], List[List[int]]]:
        single = isinstance(text, str)
        batch = [text] if single else list(text)
        out = []
        for t in batch:
            ids = self._encode_one(t, **kw)
            if add_bos:
                ids = [self.bos_token_id] + ids
            if add_eos:
                ids = ids + [self.eos_token_id]
            if max_length is not None and truncation:
                ids = ids[:max_length]
            out.append(ids)
        if padding and max_length is not None:
            out = [ids + [self.pad_token_id] * max(0, max_length - len(ids)) for ids in out]
        return out[0] if single else out

    def decode(self, ids: Union[int, List[int]], skip_special_tokens: bool = True, **kw) -> str:
        ids = [ids] if isinstance(ids, int) else list(ids)
        if skip_special_tokens:
            special = {self.bos_token_id, self.eos_token_id, self.pad_token_id} | self.THINKING_TOKEN_IDS
            ids = [t for t in ids if t not in special]
        return self._decode_ids(ids, **kw)

    def batch_decode(self, batch_ids: List[List[int]], skip_special_tokens: bool = True, **kw) -> List[str]:
        return [self.decode(i, skip_special_tokens=skip_special_tokens, **kw) for i in batch_ids]

    @property
    def bos_token(self) -> str:
        return (self._tokenizer.bos_token or "<s>") if self._tokenizer is not None else self._bos

    @property
    def eos_token(self) -> str:
        return (self._tokenizer.eos_token or "</s>") if self._tokenizer is not None else self._eos

    @property
    def pad_token(self) -> str:
        return (self._tokenizer.pad_token or "<pad>") if self._tokenizer is not None else self._pad

    def get_thinking_token_ids(self) -> Dict[str, int]:
        return {"think_start": 3, "think_end": 4, "answer_start": 5, "answer_end": 6, "summary_start": 7}

    def add_thinking_tokens(self, vocab_size: int) -> int:
        return max(vocab_size, self.SUMMARY_START_ID + 1)

    def __len__(self) -> int:
        return self.vocab_size

    def __call__(self, text, **kw):
        return {"input_ids": self.encode(text, **kw)}


def load_tokenizer(pretrained_name: str = "meta-llama/Llama-2-7b-hf", expected_vocab_size: int = 0,
                   **kwargs) -> MamformerTokenizer:
    """HuggingFace tokenizer by name or local path; falls back to the char-level tokenizer."""
    try:
        from transformers import AutoTokenizer
        tok = MamformerTokenizer(AutoTokenizer.from_pretrained(pretrained_name, **kwargs))
        if expected_vocab_size > 0 and tok.vocab_size != expected_vocab_size:
            logging.warning("Tokenizer vocab (%d) does not match model vocab (%d).",
                            tok.vocab_size, expected_vocab_size)
        return tok
    except Exception as e:  # no network here: fall back
        logging.warning("Failed to load tokenizer %r (%s); using the char-level fallback.", pretrained_name, e)
        return MamformerTokenizer()
