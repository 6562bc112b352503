"""Loss masks for multi-turn chat data: train on the assistant turns' content only.

`multi_turn_loss_mask(tokenizer, messages)` renders the conversation with the tokenizer's chat
template one message at a time. The tokens a message adds are attributed to it; for an
assistant message the generation prompt (the assistant header the template adds before the
model speaks) gets mask 0 and the rest (content and end-of-turn) gets mask 1. Templates that
re-render earlier turns differently once a later turn is appended are rejected (the token
prefix must be stable), since the mask would otherwise not line up with the tokens.

Reference: miles/utils/mask_utils.py:9-187 (MultiTurnLossMaskGenerator).
"""
from __future__ import annotations


def _render(tok, messages, add_generation_prompt: bool, tools=None) -> list[int]:
    kw = {"tools": tools} if tools else {}
    out = tok.apply_chat_template(messages, tokenize=True, add_generation_prompt=add_generation_prompt, **kw)
    return list(out["input_ids"] if isinstance(out, dict) else out)


def multi_turn_loss_mask(tokenizer, messages: list[dict], tools=None) -> tuple[list[int], list[int]]:
    ids: list[int] = []
    mask: list[int] = []
    for k, msg in enumerate(messages):
        full = _render(tokenizer, messages[:k + 1], False, tools)
        if full[:len(ids)] != ids:
            raise ValueError("chat template is not prefix-stable across turns; cannot build a "
                             "per-turn loss mask")
        new = full[len(ids):]
        if msg.get("role") == "assistant":
            head = _render(tokenizer, messages[:k], True, tools) if k else []
            h = max(0, len(head) - len(ids)) if head[:len(ids)] == ids else 0
            h = min(h, len(new))
            mask += [0] * h + [1] * (len(new) - h)
        else:
            mask += [0] * len(new)
        ids = full
    return ids, mask
