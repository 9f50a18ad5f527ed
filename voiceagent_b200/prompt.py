"""Prompt layout for Qwen3-ASR without a tokenizer.

The chat template reduces to a fixed 16-token layout with one ``<|audio_pad|>``
placeholder (prompt.py:97-142 of the reference; ids pinned by its
tests/test_prompt.py:24-47):

    <|im_start|>system\\n<|im_end|>\\n<|im_start|>user\\n<|audio_start|><|audio_pad|>
    <|audio_end|><|im_end|>\\n<|im_start|>assistant\\n

The placeholder expands to one id per audio token. A forced language appends
``language {Name}<asr_text>``; ``<asr_text>`` is 151704, while the ids of the words
``language`` and ``{Name}`` come from the checkpoint's tokenizer, which is not
available offline -- fixed placeholder ids stand in for them (three suffix tokens,
like the reference's). A system context must be given pre-tokenized.
"""

from __future__ import annotations

from dataclasses import dataclass

IM_START, IM_END, NEWLINE = 151644, 151645, 198
SYSTEM, USER, ASSISTANT = 8948, 872, 77091
AUDIO_START, AUDIO_PAD, AUDIO_END = 151669, 151676, 151670
ASR_TEXT = 151704
TEMPLATE = [IM_START, SYSTEM, NEWLINE, IM_END, NEWLINE, IM_START, USER, NEWLINE, AUDIO_START,
            AUDIO_PAD, AUDIO_END, IM_END, NEWLINE, IM_START, ASSISTANT, NEWLINE]
SYSTEM_CONTEXT_AT = 3  # context ids go between "system\n" and <|im_end|>

LANGUAGE_ALIASES = {
    "en": "English", "english": "English", "zh": "Chinese", "zh-cn": "Chinese",
    "chinese": "Chinese", "zh-tw": "Cantonese", "cantonese": "Cantonese", "ja": "Japanese",
    "ko": "Korean", "de": "German", "fr": "French", "es": "Spanish", "pt": "Portuguese",
    "it": "Italian", "ru": "Russian", "ar": "Arabic", "th": "Thai", "vi": "Vietnamese",
    "id": "Indonesian", "tr": "Turkish", "hi": "Hindi",
}
# Placeholder ids (tokenizer unavailable): "language" and one id per language name.
LANGUAGE_WORD_ID = 11528
_LANGUAGE_NAMES = sorted(set(LANGUAGE_ALIASES.values()))
LANGUAGE_NAME_IDS = {name: 12000 + i for i, name in enumerate(_LANGUAGE_NAMES)}


def normalize_language(language: str | None) -> str | None:
    if language is None:
        return None
    key = str(language).strip()
    if not key:
        return None
    return LANGUAGE_ALIASES.get(key.lower(), key[:1].upper() + key[1:].lower())


@dataclass
class PromptLayout:
    token_ids: list[int]
    audio_offset: int
    audio_length: int

    def __len__(self) -> int:
        return len(self.token_ids)


class PromptBuilder:
    def __init__(self, audio_token_id: int = AUDIO_PAD, stop_token_ids=(151643, 151645)):
        self.audio_token_id = audio_token_id
        self.stop_token_ids = set(stop_token_ids)

    def template(self, context_ids: list[int] | None = None, language: str | None = None):
        ids = list(TEMPLATE)
        if context_ids:
            ids[SYSTEM_CONTEXT_AT:SYSTEM_CONTEXT_AT] = list(context_ids)
        if language:
            name_id = LANGUAGE_NAME_IDS.get(language, 12000 + len(_LANGUAGE_NAMES)
                                            + sum(map(ord, language)) % 1000)
            ids += [LANGUAGE_WORD_ID, name_id, ASR_TEXT]
        return ids, ids.index(self.audio_token_id)

    def build(self, num_audio_tokens: int, context: str | list[int] = "",
              language: str | None = None) -> PromptLayout:
        if num_audio_tokens < 1:
            raise ValueError(f"num_audio_tokens must be positive, got {num_audio_tokens}")
        if isinstance(context, str):
            if context:
                raise ValueError("no tokenizer is available offline: pass the system context "
                                 "as a list of token ids")
            context = []
        ids, off = self.template(list(context), language)
        token_ids = ids[:off] + [self.audio_token_id] * num_audio_tokens + ids[off + 1:]
        return PromptLayout(token_ids=token_ids, audio_offset=off, audio_length=num_audio_tokens)

    def decode(self, token_ids: list[int]) -> str:
        """No tokenizer offline: the raw text is the id sequence itself."""
        return " ".join(str(t) for t in token_ids)
