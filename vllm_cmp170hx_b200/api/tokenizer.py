"""Tokenizers: a local Hugging Face tokenizer when a path is given (offline,
``local_files_only``), else a byte-level tokenizer (UTF-8 bytes + a few
special tokens) that serves random-init models end to end.

Chat rendering includes system messages inline, the behaviour of the
reference's DeepSeek-V4.1 tokenizer registration for Anthropic
``/v1/messages`` (vllm_sm80/tokenizers/deepseek_v41.py).
"""

from __future__ import annotations


class ByteTokenizer:
    SPECIALS = ["<|bos|>", "<|eos|>", "<|pad|>", "<|system|>", "<|user|>", "<|assistant|>", "<|tool|>"]

    def __init__(self, vocab_size: int = 512):
        self.offset = len(self.SPECIALS)
        assert vocab_size >= 256 + self.offset
        self.vocab_size = vocab_size
        self.special_ids = {t: i for i, t in enumerate(self.SPECIALS)}
        self.bos_token_id = 0
        self.eos_token_id = 1

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        ids = [b + self.offset for b in text.encode("utf-8")]
        return ([self.bos_token_id] if add_bos else []) + ids

    def decode(self, ids: list[int], skip_special: bool = True) -> str:
        out = bytearray()
        for i in ids:
            i = int(i) % self.vocab_size
            if i < self.offset:
                if not skip_special:
                    out += self.SPECIALS[i].encode()
                continue
            b = i - self.offset
            if b < 256:
                out.append(b)
        return out.decode("utf-8", errors="replace")

    def apply_chat_template(self, messages: list[dict], add_generation_prompt: bool = True) -> list[int]:
        ids = [self.bos_token_id]
        for m in messages:
            role = m.get("role", "user")
            tag = {"system": "<|system|>", "assistant": "<|assistant|>", "tool": "<|tool|>"}.get(role, "<|user|>")
            ids.append(self.special_ids[tag])
            content = m.get("content") or ""
            if isinstance(content, list):  # Anthropic / OpenAI content blocks
                content = "".join(b.get("text", "") for b in content if isinstance(b, dict))
            ids += self.encode(content)
        if add_generation_prompt:
            ids.append(self.special_ids["<|assistant|>"])
        return ids


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True, trust_remote_code=False)
        self.eos_token_id = self.tok.eos_token_id
        self.vocab_size = len(self.tok)

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        return self.tok.encode(text, add_special_tokens=add_bos)

    def decode(self, ids, skip_special: bool = True) -> str:
        return self.tok.decode(ids, skip_special_tokens=skip_special)

    def apply_chat_template(self, messages, add_generation_prompt: bool = True) -> list[int]:
        return self.tok.apply_chat_template(messages, add_generation_prompt=add_generation_prompt, tokenize=True)


def get_tokenizer(path: str | None, vocab_size: int):
    return HFTokenizer(path) if path else ByteTokenizer(vocab_size)
