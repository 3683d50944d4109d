"""Character-level tokenizer with chat special tokens (tokenizer.py:1-74).

Ids: 8 specials, then the 95 printable ASCII characters (32..126), then newline;
vocab 104.  The id order is part of the rollout format, so it matches the reference.
"""

from __future__ import annotations

SPECIAL_TOKENS = ["<pad>", "<bos>", "<eos>", "<unk>", "<|system|>", "<|user|>", "<|assistant|>", "<|end|>"]
BOUNDARY_TOKENS = {"<bos>", "<|system|>", "<|user|>", "<|assistant|>", "<|end|>"}


class CharTokenizer:
    def __init__(self) -> None:
        self.itos: list[str] = SPECIAL_TOKENS + [chr(c) for c in range(32, 127)] + ["\n"]
        self.stoi: dict[str, int] = {s: i for i, s in enumerate(self.itos)}
        self.special_ids = {self.stoi[s] for s in SPECIAL_TOKENS}
        self.boundary_ids = {self.stoi[s] for s in BOUNDARY_TOKENS}

    @property
    def vocab_size(self) -> int:
        return len(self.itos)

    @property
    def pad_id(self) -> int:
        return self.stoi["<pad>"]

    @property
    def bos_id(self) -> int:
        return self.stoi["<bos>"]

    @property
    def eos_id(self) -> int:
        return self.stoi["<eos>"]

    @property
    def unk_id(self) -> int:
        return self.stoi["<unk>"]

    @property
    def end_id(self) -> int:
        return self.stoi["<|end|>"]

    def role_id(self, role: str) -> int:
        return self.stoi[f"<|{role}|>"]

    def encode(self, text: str) -> list[int]:
        return [self.stoi.get(ch, self.unk_id) for ch in text]

    def decode(self, ids, skip_special: bool = True) -> str:
        chars = []
        for i in ids:
            i = int(i)
            if skip_special and i in self.special_ids:
                continue
            chars.append(self.itos[i])
        return "".join(chars)

    def is_boundary(self, token_id: int) -> bool:
        return int(token_id) in self.boundary_ids
