"""Token-in-token-out (TITO) tokenization of multi-turn trajectories.

A multi-turn agent trajectory must be trained on exactly the tokens the engine produced and
consumed. Re-rendering the whole conversation with the chat template after each turn does not
give those tokens when the template is not prefix-stable: thinking templates drop earlier
turns' reasoning, some templates re-render tool calls, and the generated turn ends with an
end-of-turn token while the template's rendering of that turn ends with more (a newline).

`IncrementalTokenizer` extends a token prefix (prompt + every generated token so far) with the
tokens of the messages appended after the last assistant turn, rendering each appended segment
in a small synthetic context instead of the real history:

  * a run of consecutive `tool` messages behind [system, assistant-with-matching-tool-calls],
  * each `user` / `system` message behind [system],

keeping only the tokens the segment adds to its context, then the generation prompt of the
next assistant turn. At the junction with the prefix it adds whatever the template renders after
an assistant turn's content that the generation did not produce (e.g. the newline after the
end-of-turn token; all of it when the turn hit the length limit).

`TokenSeqComparator` explains how two token sequences of one conversation differ (for
example the incremental sequence against a full re-render): it splits both at the template's
special tokens and reports structural differences, differences in non-assistant text, and
differences inside assistant turns (expected where a template rewrites earlier turns).

Reference roles: miles/utils/chat_template_utils/tito_tokenizer.py (incremental tokenization with
synthetic prefixes, per-model junction fixes), token_seq_comparator.py (segment comparison).
"""
from __future__ import annotations

from dataclasses import dataclass, field

_SYSTEM = {"role": "system", "content": "You are a helpful assistant."}
_MARK = "TITOMARKER"


def _ids(out) -> list[int]:
    if isinstance(out, dict):
        out = out["input_ids"]
    return [int(t) for t in out]


class IncrementalTokenizer:
    def __init__(self, tokenizer, tools=None):
        self.tok = tokenizer
        self.tools = tools
        self._tail: list[int] | None = None

    # ------------------------------------------------------------------ rendering
    def render(self, messages: list[dict], add_generation_prompt: bool = False) -> list[int]:
        kw = {"tools": self.tools} if self.tools else {}
        return _ids(self.tok.apply_chat_template(messages, tokenize=True,
                                                 add_generation_prompt=add_generation_prompt, **kw))

    def _delta(self, ctx: list[dict], full: list[dict]) -> list[int]:
        a, b = self.render(ctx), self.render(full)
        if b[:len(a)] != a:
            raise ValueError("the chat template renders the synthetic context differently when "
                             "messages follow it; it cannot be tokenized incrementally")
        return b[len(a):]

    @staticmethod
    def _assistant_for(tools: list[dict]) -> dict:
        """An assistant turn whose tool calls match the tool responses that follow it."""
        return {"role": "assistant", "content": "",
                "tool_calls": [{"id": t.get("tool_call_id") or f"call_{i}", "type": "function",
                                "function": {"name": t.get("name") or "tool", "arguments": {}}}
                               for i, t in enumerate(tools)]}

    # ------------------------------------------------------------------ pieces
    def turn_tail(self) -> list[int]:
        """Tokens the template renders after an assistant turn's content (end-of-turn token and
        separator), found by rendering a marker turn and taking what follows the marker."""
        if self._tail is None:
            if not hasattr(self.tok, "encode"):  # cannot locate the content: no junction
                self._tail = []
                return self._tail
            ids = self.render([_SYSTEM, {"role": "user", "content": "q"},
                               {"role": "assistant", "content": _MARK}])
            mark = _ids(self.tok.encode(_MARK, add_special_tokens=False))
            pos = -1
            for i in range(len(ids) - len(mark), -1, -1):
                if ids[i:i + len(mark)] == mark:
                    pos = i + len(mark)
                    break
            self._tail = ids[pos:] if pos >= 0 else []
        return self._tail

    def suffix(self, appended: list[dict]) -> list[int]:
        """Tokens of the messages appended after the last assistant turn, plus the next
        assistant turn's generation prompt."""
        out: list[int] = []
        i = 0
        while i < len(appended):
            m = appended[i]
            if m.get("role") == "assistant":
                raise ValueError("appended messages must not contain assistant turns")
            if m.get("role") == "tool":
                j = i
                while j < len(appended) and appended[j].get("role") == "tool":
                    j += 1
                ctx = [_SYSTEM, self._assistant_for(appended[i:j])]
                out += self._delta(ctx, ctx + appended[i:j])
                i = j
            else:
                out += self._delta([_SYSTEM], [_SYSTEM, m])
                i += 1
        ctx = [_SYSTEM, {"role": "user", "content": "q"}]
        with_prompt, without = self.render(ctx, True), self.render(ctx, False)
        if with_prompt[:len(without)] != without:
            raise ValueError("the generation prompt is not an extension of the rendering")
        return out + with_prompt[len(without):]

    def junction(self, prefix: list[int]) -> list[int]:
        """Tokens to add after a generated assistant turn so that it ends the way the template
        ends an assistant turn: the part of the turn tail the generation did not emit."""
        tail = self.turn_tail()
        for k in range(min(len(tail), len(prefix)), 0, -1):
            if prefix[-k:] == tail[:k]:
                return tail[k:]
        return list(tail)

    def extend(self, prefix: list[int], appended: list[dict]) -> list[int]:
        """prefix (prompt + generated tokens, ending with the last assistant turn) followed by
        the appended messages and the next generation prompt."""
        return list(prefix) + self.junction(prefix) + self.suffix(appended)


# ---------------------------------------------------------------------------------- comparator
@dataclass
class Segment:
    special: int | None          # the special token that opens the segment (None: start)
    tokens: list[int] = field(default_factory=list)


@dataclass
class Mismatch:
    kind: str      # "structure" | "text" | "assistant_text"
    index: int     # segment index
    detail: str


class TokenSeqComparator:
    def __init__(self, tokenizer, special_ids: set[int] | None = None,
                 assistant_marker_ids: list[int] | None = None):
        """special_ids: ids that delimit segments (default: the tokenizer's special tokens);
        assistant_marker_ids: tokens that open an assistant turn's segment, e.g. the encoding of
        the assistant role header (default: none, every content difference counts as text)."""
        self.tok = tokenizer
        if special_ids is None:
            special_ids = set(getattr(tokenizer, "all_special_ids", []) or [])
            added = getattr(tokenizer, "added_tokens_decoder", None)
            if added:
                special_ids |= {int(i) for i, t in added.items() if getattr(t, "special", False)}
        self.special = set(special_ids)
        self.assistant_marker = assistant_marker_ids

    def segments(self, ids: list[int]) -> list[Segment]:
        out = [Segment(None)]
        for t in ids:
            if t in self.special:
                out.append(Segment(t))
            else:
                out[-1].tokens.append(t)
        return out

    def _is_assistant(self, seg: Segment) -> bool:
        m = self.assistant_marker
        return bool(m) and seg.tokens[:len(m)] == m

    def compare(self, expected: list[int], actual: list[int]) -> list[Mismatch]:
        a, b = self.segments(expected), self.segments(actual)
        out: list[Mismatch] = []
        if [s.special for s in a] != [s.special for s in b]:
            out.append(Mismatch("structure", -1, f"special-token sequences differ: {len(a)} vs {len(b)} segments"))
            return out
        for i, (x, y) in enumerate(zip(a, b)):
            if x.tokens == y.tokens:
                continue
            kind = "assistant_text" if (self._is_assistant(x) or self._is_assistant(y)) else "text"
            out.append(Mismatch(kind, i, f"segment {i}: {len(x.tokens)} vs {len(y.tokens)} tokens"))
        return out
