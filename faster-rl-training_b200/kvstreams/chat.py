"""Chat layout of a rollout stream (chat.py:1-38)::

    <bos><|system|>...<|end|> pads          prompt segment (protected)
    <|user|>...<|end|><|assistant|>...<|end|> pads    one turn

With padding to the block size every segment occupies whole KV blocks.
"""

from __future__ import annotations

from .tokenizer import CharTokenizer


class ChatTemplate:
    def __init__(self, tokenizer: CharTokenizer) -> None:
        self.tok = tokenizer

    def system(self, text: str) -> list[int]:
        return [self.tok.bos_id, self.tok.role_id("system")] + self.tok.encode(text) + [self.tok.end_id]

    def user_turn(self, text: str) -> list[int]:
        """User message plus the assistant header the model continues from."""
        return [self.tok.role_id("user")] + self.tok.encode(text) + [self.tok.end_id, self.tok.role_id("assistant")]

    def assistant_end(self) -> list[int]:
        return [self.tok.end_id]

    def padding(self, stream_len: int, block_size: int) -> list[int]:
        return [self.tok.pad_id] * ((-stream_len) % block_size)
