"""Synthetic tokenizer for seeded workloads (no real MiniMind-IME tokenizer or
checkpoint is available offline).

Ids: 0 pad, 1 BOS, 2 EOS, 3..9 the terminal punctuation "。！？；!?;" (so the
engine's terminal-stop and decoded-terminal logic is exercised), and every id
>= 10 is one CJK character, ``chr(0x4E00 + id - 10)``. ``decode(encode(s)) == s``
for any string of those characters, which the refill exact-repeat bans rely on.
Characters outside the vocabulary are dropped by ``encode``.
"""

from __future__ import annotations

from collections.abc import Iterable, Sequence

TERMINALS = "。！？；!?;"
CJK_BASE = 0x4E00
FIRST_CJK_ID = 3 + len(TERMINALS)


class SyntheticTokenizer:
    pad_token_id = 0
    bos_token_id = 1
    eos_token_id = 2

    def __init__(self, vocab_size: int):
        if vocab_size <= FIRST_CJK_ID:
            raise ValueError("vocab_size too small for the synthetic tokenizer")
        self.vocab_size = vocab_size
        self._punct = {ch: 3 + i for i, ch in enumerate(TERMINALS)}
        # decode table: the text of every id, "" for the special ids
        self._table = ["", "", ""] + [self.id_to_char(i) for i in range(3, vocab_size)]

    def id_to_char(self, token_id: int) -> str:
        if 3 <= token_id < FIRST_CJK_ID:
            return TERMINALS[token_id - 3]
        if FIRST_CJK_ID <= token_id < self.vocab_size:
            return chr(CJK_BASE + token_id - FIRST_CJK_ID)
        return ""

    def char_to_id(self, ch: str) -> int | None:
        if ch in self._punct:
            return self._punct[ch]
        token_id = ord(ch) - CJK_BASE + FIRST_CJK_ID
        if FIRST_CJK_ID <= token_id < self.vocab_size:
            return token_id
        return None

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        ids = [i for i in (self.char_to_id(ch) for ch in text) if i is not None]
        if add_special_tokens:
            ids = [self.bos_token_id, *ids]
        return ids

    def decode(self, ids: Iterable[int], skip_special_tokens: bool = True, clean_up_tokenization_spaces: bool = False) -> str:
        if skip_special_tokens:
            table, vocab = self._table, self.vocab_size
            return "".join([table[i] if 0 <= i < vocab else "" for i in map(int, ids)])
        out = []
        for token_id in ids:
            token_id = int(token_id)
            if token_id < 3:
                if not skip_special_tokens:
                    out.append(("<pad>", "<s>", "</s>")[token_id])
                continue
            out.append(self.id_to_char(token_id))
        return "".join(out)

    def batch_decode(self, sequences: Sequence[Iterable[int]], skip_special_tokens: bool = True,
                     clean_up_tokenization_spaces: bool = False) -> list[str]:
        return [self.decode(s, skip_special_tokens, clean_up_tokenization_spaces) for s in sequences]

    def text_for(self, ids: Iterable[int]) -> str:
        """Inverse of ``encode`` for ids >= 3 (used to build prefixes from ids)."""
        return "".join(self.id_to_char(int(i)) for i in ids)
