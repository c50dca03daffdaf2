"""Tokenizers for the server: a byte-level one that needs no files (ids 0..2 = pad/bos/eos, 3..258 = bytes), or a
Hugging Face tokenizer loaded from a local directory."""
from __future__ import annotations


class ByteTokenizer:
    pad_id, bos_id, eos_id = 0, 1, 2
    vocab_size = 259

    def encode(self, text: str) -> list[int]:
        return [b + 3 for b in text.encode("utf-8")]

    def decode(self, ids: list[int]) -> str:
        return bytes((i - 3) % 256 for i in ids if i >= 3).decode("utf-8", errors="replace")

    def chat(self, messages: list[dict]) -> list[int]:
        text = "".join(f"<|{m.get('role', 'user')}|>{_content_text(m.get('content', ''))}\n" for m in messages)
        return self.encode(text + "<|assistant|>")


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_id = self.tok.eos_token_id

    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text, add_special_tokens=False)

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    def chat(self, messages: list[dict]) -> list[int]:
        msgs = [{"role": m.get("role", "user"), "content": _content_text(m.get("content", ""))} for m in messages]
        return self.tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=True)


def _content_text(content) -> str:
    """OpenAI content is a string or a list of parts ({"type": "text"|"input_text", "text": ...})."""
    if isinstance(content, str):
        return content
    return "".join(p.get("text", "") for p in content if isinstance(p, dict))
