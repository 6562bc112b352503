"""TITO tokenization: incremental suffixes for appended tool / user turns, the junction after a
generated assistant turn, the fallback for templates that are not prefix-stable (a thinking
template that drops earlier reasoning), and the segment comparator."""
from miles_b200.rollout.session import Session
from miles_b200.rollout.tito import IncrementalTokenizer, TokenSeqComparator

SPECIAL = {"<s>": 1, "<e>": 2}  # turn start / end tokens


class _ThinkTok:
    """Word-level tokenizer with a Qwen-like template: each turn is <s>role text<e> followed by a
    newline; assistant turns render their reasoning only when they are the last turn (earlier
    reasoning is dropped, so the template is not prefix-stable)."""

    def __init__(self):
        self.vocab = dict(SPECIAL)
        self.vocab["\\n"] = 3

    def _id(self, w):
        if w not in self.vocab:
            self.vocab[w] = len(self.vocab) + 10
        return self.vocab[w]

    def encode(self, text, add_special_tokens=False):
        out = []
        for w in text.replace("\\n", " \\n ").split():
            out.append(self._id(w))
        return out

    def apply_chat_template(self, messages, tools=None, tokenize=False, add_generation_prompt=False, **kw):
        ids = []
        last_asst = max((i for i, m in enumerate(messages) if m["role"] == "assistant"), default=-1)
        for i, m in enumerate(messages):
            ids.append(SPECIAL["<s>"])
            ids += self.encode(m["role"])
            if m["role"] == "assistant" and m.get("reasoning") and i == last_asst:
                ids += self.encode("think " + m["reasoning"])
            if m["role"] == "tool":
                ids += self.encode("result")
            ids += self.encode(m.get("content") or "")
            ids.append(SPECIAL["<e>"])
            ids.append(3)  # newline
        if add_generation_prompt:
            ids += [SPECIAL["<s>"]] + self.encode("assistant")
        return ids


def test_suffix_and_junction():
    tok = _ThinkTok()
    tito = IncrementalTokenizer(tok)
    assert tito.turn_tail() == [SPECIAL["<e>"], 3]
    gen = tok.encode("assistant think hmm answer") + [SPECIAL["<e>"]]  # engine stops at <e>
    assert tito.junction(gen) == [3]
    assert tito.junction(gen[:-1]) == [SPECIAL["<e>"], 3]  # length-limited turn
    tools = [{"role": "tool", "content": "42"}, {"role": "tool", "content": "7"}]
    suf = tito.suffix(tools + [{"role": "user", "content": "more"}])
    expect = []
    for c in ("42", "7"):
        expect += [SPECIAL["<s>"]] + tok.encode(f"tool result {c}") + [SPECIAL["<e>"], 3]
    expect += [SPECIAL["<s>"]] + tok.encode("user more") + [SPECIAL["<e>"], 3]
    expect += [SPECIAL["<s>"]] + tok.encode("assistant")
    assert suf == expect


def test_session_uses_incremental_path_when_not_prefix_stable():
    tok = _ThinkTok()
    s = Session()
    msgs = [{"role": "user", "content": "hi"}]
    ids, mask, lps = s.prepare(tok, msgs)
    out_ids = tok.encode("think hmm answer") + [SPECIAL["<e>"]]  # generated, reasoning included
    reply = {"role": "assistant", "content": "answer", "reasoning": "hmm"}
    s.commit(msgs, reply, ids, mask, lps, out_ids, [-0.5] * len(out_ids))
    msgs2 = msgs + [reply, {"role": "tool", "content": "42"}]
    ids2, mask2, _ = s.prepare(tok, msgs2, allowed_roles=["tool"])
    # the generated tokens (with the reasoning the template would drop) are kept verbatim
    assert ids2[:len(ids) + len(out_ids)] == ids + out_ids
    rest = ids2[len(ids) + len(out_ids):]
    assert rest == [3] + [SPECIAL["<s>"]] + tok.encode("tool result 42") + [SPECIAL["<e>"], 3] + \
        [SPECIAL["<s>"]] + tok.encode("assistant")
    assert mask2 == mask + [1] * len(out_ids) + [0] * len(rest)


def test_comparator_classifies_differences():
    tok = _ThinkTok()
    comp = TokenSeqComparator(tok, special_ids=set(SPECIAL.values()),
                              assistant_marker_ids=tok.encode("assistant"))
    full = tok.apply_chat_template([{"role": "user", "content": "hi"},
                                    {"role": "assistant", "content": "a", "reasoning": "r"},
                                    {"role": "user", "content": "x"}])
    inc = tok.apply_chat_template([{"role": "user", "content": "hi"},
                                   {"role": "assistant", "content": "a"},
                                   {"role": "user", "content": "x"}])
    assert comp.compare(full, full) == []
    # the last assistant turn keeps its reasoning in one render only: an assistant-text difference
    assert [m.kind for m in comp.compare(full, inc)] == ["assistant_text"]
    bad = list(inc)
    bad[bad.index(tok.vocab["x"])] = tok.vocab["hi"]
    assert [m.kind for m in comp.compare(inc, bad)] == ["text"]
    assert [m.kind for m in comp.compare(inc, inc[:-2])] == ["structure"]
