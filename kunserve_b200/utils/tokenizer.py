"""Tokenizer wrapper and incremental detokenization (parity:
``kunserve/tokenizer.py:16-123``).  Tokenizers load from local files only."""
from typing import List, Optional, Tuple


def get_tokenizer(name: str, tokenizer_mode: str = "auto", trust_remote_code: bool = False):
    from transformers import AutoTokenizer

    return AutoTokenizer.from_pretrained(name, use_fast=tokenizer_mode != "slow",
                                         trust_remote_code=trust_remote_code, local_files_only=True)


def detokenize_incrementally(tokenizer, all_ids: List[int], prev_tokens: Optional[List[str]],
                             prefix_offset: int = 0, read_offset: int = 0,
                             skip_special_tokens: bool = False) -> Tuple[List[str], str, int, int]:
    """Decode only what the newest id adds: returns (new tokens, new text,
    prefix offset, read offset).  Text is held back while the tail is an
    incomplete UTF-8 sequence (decodes to U+FFFD)."""
    new_id = all_ids[-1]
    if prev_tokens is None:
        toks = tokenizer.convert_ids_to_tokens(all_ids, skip_special_tokens=skip_special_tokens)
        prev_tokens = toks[:-1]
        new_tokens = toks[-1:]
        prefix_offset = max(len(prev_tokens) - 5, 0)
        read_offset = len(prev_tokens)
    else:
        new_tokens = tokenizer.convert_ids_to_tokens([new_id], skip_special_tokens=skip_special_tokens)
    out_tokens = prev_tokens + new_tokens
    prefix = tokenizer.convert_tokens_to_string(out_tokens[prefix_offset:read_offset])
    full = tokenizer.convert_tokens_to_string(out_tokens[prefix_offset:])
    if len(full) > len(prefix) and not full.endswith("�"):
        return new_tokens, full[len(prefix):], read_offset, len(out_tokens)
    return new_tokens, "", prefix_offset, read_offset
