"""Tokenizers for the server.

Random-init checkpoints have no vocabulary, so the default is a byte-level
tokenizer: UTF-8 bytes map to ids 3..258 (0 = pad, 1 = bos, 2 = eos), and
ids outside the byte range decode to ``<|id|>`` placeholders. A checkpoint
that ships a HuggingFace tokenizer directory loads it with ``transformers``
(offline, ``local_files_only``).
"""
from __future__ import annotations

import os


class ByteTokenizer:
    OFFSET = 3
    pad_token_id, bos_token_id, eos_token_id = 0, 1, 2

    def __init__(self, vocab_size: int = 151936):
        self.vocab_size = vocab_size

    def encode(self, text: str) -> list[int]:
        return [b + self.OFFSET for b in text.encode("utf-8")]

    def decode(self, ids) -> str:
        out = bytearray()
        parts: list[str] = []
        for t in ids:
            t = int(t)
            if self.OFFSET <= t < self.OFFSET + 256:
                out.append(t - self.OFFSET)
            else:
                if out:
                    parts.append(out.decode("utf-8", errors="replace"))
                    out = bytearray()
                if t not in (self.pad_token_id, self.bos_token_id, self.eos_token_id):
                    parts.append("<|%d|>" % t)
        if out:
            parts.append(out.decode("utf-8", errors="replace"))
        return "".join(parts)

    def apply_chat_template(self, messages: list[dict]) -> list[int]:
        text = "".join("<|%s|>\n%s\n" % (m.get("role", "user"), _content(m)) for m in messages)
        return self.encode(text + "<|assistant|>\n")


class IncrementalDecoder:
    """Text deltas of a growing token list, for streaming.

    Decoding each delta alone splits multi-byte characters (and, for
    subword tokenizers, spacing that depends on the previous token). Instead
    the window of tokens since the last emission is decoded twice, with and
    without the new tokens, and the difference is emitted; while the window
    ends in an incomplete character (U+FFFD), nothing is emitted until more
    tokens complete it or the stream ends. The concatenated deltas equal one
    decode of all tokens."""

    def __init__(self, tokenizer):
        self.tok = tokenizer
        self.ids: list[int] = []
        self.prefix = 0  # window start: tokens before it are emitted for good
        self.read = 0    # tokens up to here are emitted

    def push(self, new, final: bool = False) -> str:
        self.ids.extend(int(t) for t in new)
        before = self.tok.decode(self.ids[self.prefix:self.read])
        now = self.tok.decode(self.ids[self.prefix:])
        if len(now) > len(before) and (final or not now.endswith("\ufffd")):
            self.prefix, self.read = self.read, len(self.ids)
            return now[len(before):]
        if final:
            self.prefix = self.read = len(self.ids)
            return now[len(before):]
        return ""


def _content(m: dict) -> str:
    c = m.get("content", "")
    if isinstance(c, list):  # OpenAI content parts: keep the text parts
        return "".join(p.get("text", "") for p in c if isinstance(p, dict))
    return str(c)


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_token_id = self.tok.eos_token_id

    def encode(self, text: str) -> list[int]:
        return list(self.tok.encode(text, add_special_tokens=False))

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)

    def apply_chat_template(self, messages: list[dict]) -> list[int]:
        msgs = [{"role": m.get("role", "user"), "content": _content(m)} for m in messages]
        return list(self.tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=True))


def load_tokenizer(path: str | None, vocab_size: int):
    if path and os.path.isdir(path):
        return HFTokenizer(path)
    return ByteTokenizer(vocab_size)


class StopMatcher:
    """Stop strings over streamed text (the OpenAI ``stop`` field).

    Text is fed as it is decoded; ``feed`` returns what may be shown now and
    whether a stop string was met. Up to ``len(longest stop) - 1`` trailing
    characters are held back, because they may be the start of a stop string
    that the next tokens complete; text from the first stop string on is
    never shown. Without stop strings the text passes through unchanged."""

    def __init__(self, stops=None, include: bool = False):
        if isinstance(stops, str):
            stops = [stops]
        self.stops = [s for s in (stops or []) if s]
        self.include = include  # vLLM's include_stop_str_in_output: the matched string is shown too
        self.hold = max((len(s) for s in self.stops), default=1) - 1
        self.buf = ""
        self.done = False

    def feed(self, text: str, final: bool = False) -> tuple[str, bool]:
        if self.done:
            return "", True
        self.buf += text
        hits = [(i, len(s)) for i, s in ((self.buf.find(s), s) for s in self.stops) if i >= 0]
        if hits:
            at, n = min(hits)
            out, self.buf, self.done = self.buf[:at + (n if self.include else 0)], "", True
            return out, True
        if final or self.hold == 0:
            out, self.buf = self.buf, ""
            return out, False
        cut = max(0, len(self.buf) - self.hold)
        out, self.buf = self.buf[:cut], self.buf[cut:]
        return out, False
