"""Prompt formatting: ChatML with Qwen3 "thinking" mode, benchmark suffixes.

Behaviour (and the exact instruction strings, which benchmark graders match
on) follows ``pio/common/processing/prompt_utils.py:9-91``: math prompts get a
step-by-step/boxed-answer instruction, multiple-choice prompts a JSON answer
instruction, assistant turns in the history lose their ``<think>...</think>``
spans, and the chat template is ChatML with an optional ``<think>`` opener.
"""
from __future__ import annotations

import re
from typing import Dict, List, Union

MATH_SUFFIX = "Please reason step by step, and put your final answer within \\boxed{}."
MCQ_SUFFIX = 'Please show your choice in the answer field with only the choice letter, e.g., "answer": "C".'
_THINK = re.compile(r"<think>.*?</think>", re.S)


def _append_once(query: str, suffix: str) -> str:
    return query if suffix in query else f"{query}\n\n{suffix}"


def format_math_prompt(query: str) -> str:
    return _append_once(query, MATH_SUFFIX)


def format_mcq_prompt(query: str) -> str:
    return _append_once(query, MCQ_SUFFIX)


def strip_thinking(text: str) -> str:
    return _THINK.sub("", text).strip()


def format_history(history: List[Dict[str, str]]) -> List[Dict[str, str]]:
    out = []
    for turn in history:
        if turn.get("role") in ("assistant", "model"):
            out.append({"role": turn["role"], "content": strip_thinking(turn.get("content", ""))})
        else:
            out.append(dict(turn))
    return out


def apply_chat_template(tokenizer, messages: List[Dict[str, str]], add_generation_prompt: bool = True,
                        enable_thinking: bool = True, tokenize: bool = False) -> Union[str, List[int]]:
    parts = [f"<|im_start|>{m.get('role', 'user')}\n{m.get('content', '')}<|im_end|>\n" for m in messages]
    text = "".join(parts)
    if add_generation_prompt:
        text += "<|im_start|>assistant\n" + ("<think>\n" if enable_thinking else "")
    if tokenize:
        return tokenizer.encode(text)
    return text
