"""Rule-based and remote reward models.

`async_rm(args, sample)` dispatches on `sample.metadata["rm_type"]` or `--rm-type`:
  deepscaler | dapo | math | f1 | gpqa | ifbench | random | remote_rm, with a `boxed_` prefix
that first extracts the last \\boxed{...} of the response; `--custom-rm-path` overrides it.
`batched_async_rm` evaluates a group (for `--group-rm`).

The graders are written from the grading rules (last boxed answer / "Answer:" line, LaTeX
normalisation, numeric equivalence with tolerance, exact string match fallback), not taken
from any particular grader implementation.

Reference: miles/rollout/rm_hub/__init__.py:17-90 (dispatch and return conventions: math and
deepscaler return 1/0, dapo returns {"score": 1/-1, "acc", "pred"}, f1 returns the F1 score).
"""
from __future__ import annotations

import asyncio
import random
import re
import string
from collections import Counter
from fractions import Fraction

from miles_b200.utils.misc import load_function
from miles_b200.utils.types import Sample


# ----------------------------------------------------------------------------- extraction
def last_boxed(text: str) -> str | None:
    """Content of the last \\boxed{...} (or \\fbox{...}) with balanced braces."""
    if not text:
        return None
    i = max(text.rfind("\\boxed"), text.rfind("\\fbox"))
    if i < 0:
        return None
    j = text.find("{", i)
    if j < 0:
        # "\boxed 5" form
        m = re.match(r"\\boxed\s+([^\s$]+)", text[i:])
        return m.group(1) if m else None
    depth = 0
    for k in range(j, len(text)):
        if text[k] == "{":
            depth += 1
        elif text[k] == "}":
            depth -= 1
            if depth == 0:
                return text[j + 1:k]
    return None


extract_boxed_answer = last_boxed


_UNITS = ["degrees", "degree", "cm", "centimeters", "meters", "m", "inches", "inch", "feet",
          "units", "unit", "sq", "square", "dollars", "\\%", "%", "\\$"]


def normalize_math(s: str) -> str:
    """Canonical string form of a final answer (LaTeX wrappers, spacing, units, fractions)."""
    if s is None:
        return ""
    s = str(s).strip()
    s = re.sub(r"\\text\{\s*([^}]*)\}", r"\1", s)
    s = re.sub(r"\\mathrm\{\s*([^}]*)\}", r"\1", s)
    s = re.sub(r"\\mbox\{\s*([^}]*)\}", r"\1", s)
    for a, b in [("\\left", ""), ("\\right", ""), ("\\!", ""), ("\\,", ""), ("\\;", ""),
                 ("\\:", ""), ("\\ ", ""), ("dfrac", "frac"), ("tfrac", "frac"), ("^\\circ", ""),
                 ("^{\\circ}", ""), ("\\displaystyle", ""), ("$", "")]:
        s = s.replace(a, b)
    s = s.strip()
    if s.endswith("."):
        s = s[:-1]
    for u in _UNITS:
        if s.endswith(u) and len(s) > len(u):
            s = s[: -len(u)].strip()
    s = re.sub(r"^[a-zA-Z]\s*=\s*", "", s)  # "x = 5" -> "5"
    s = s.replace(" ", "")
    # \frac12 -> \frac{1}{2};  \sqrt2 -> \sqrt{2}
    s = re.sub(r"\\frac(\d)(\d)", r"\\frac{\1}{\2}", s)
    s = re.sub(r"\\sqrt(\d+)", r"\\sqrt{\1}", s)
    s = re.sub(r"(\d),(\d{3})", r"\1\2", s)  # thousands separators
    if s.startswith("0.") is False and re.fullmatch(r"\.\d+", s):
        s = "0" + s
    return s


def _to_number(s: str):
    s = s.replace("{", "").replace("}", "") if s.startswith("\\frac") else s
    m = re.fullmatch(r"\\frac(-?\d+)(-?\d+)", s)
    try:
        if m:
            return Fraction(int(m.group(1)), int(m.group(2)))
        m2 = re.fullmatch(r"(-?\d+)/(\d+)", s)
        if m2:
            return Fraction(int(m2.group(1)), int(m2.group(2)))
        if "%" in s:
            return Fraction(s.replace("%", "")) / 100
        return Fraction(s)
    except (ValueError, ZeroDivisionError):
        return None


def math_equal(pred: str, gt: str) -> bool:
    a, b = normalize_math(pred), normalize_math(gt)
    if not a:
        return False
    if a == b:
        return True
    na, nb = _to_number(a), _to_number(b)
    if na is not None and nb is not None:
        return abs(float(na) - float(nb)) <= 1e-6 * max(1.0, abs(float(nb)))
    # unordered tuples / sets
    if "," in a and "," in b:
        sa = sorted(x for x in a.strip("()[]{}").split(","))
        sb = sorted(x for x in b.strip("()[]{}").split(","))
        return len(sa) == len(sb) and all(math_equal(x, y) for x, y in zip(sa, sb))
    return False


def grade_answer(response: str, label) -> bool:
    """Grade a free-form response: compare its last boxed answer (or the response itself)."""
    pred = last_boxed(response)
    if pred is None:
        pred = response
    labels = label if isinstance(label, (list, tuple)) else [label]
    return any(math_equal(pred, str(l)) for l in labels)


# ----------------------------------------------------------------------------- graders
def deepscaler_reward(response: str, label) -> int:
    """1 if the final boxed answer after the reasoning block equals the label, else 0."""
    if "</think>" in response:
        response = response.split("</think>", 1)[1]
    elif "<think>" in response:
        return 0
    ans = last_boxed(response)
    if ans is None:
        return 0
    labels = label if isinstance(label, (list, tuple)) else [label]
    for l in labels:
        l = str(l)
        if "\\boxed" in l:
            l = last_boxed(l) or l
        if math_equal(ans, l):
            return 1
    return 0


def dapo_reward(response: str, label) -> dict:
    """'Answer: X' on the last answer line, exact match after normalisation: +1 / -1."""
    tail = response[-300:]
    matches = re.findall(r"(?i)Answer\s*:\s*([^\n]+)", tail)
    pred = normalize_math(matches[-1]) if matches else ""
    ok = pred != "" and (pred == normalize_math(str(label)) or math_equal(pred, str(label)))
    return {"score": 1.0 if ok else -1.0, "acc": ok, "pred": pred}


def _f1_tokens(s: str) -> list[str]:
    s = s.lower()
    s = "".join(ch for ch in s if ch not in set(string.punctuation))
    s = re.sub(r"\b(a|an|the)\b", " ", s)
    return s.split()


def f1_score(prediction: str, ground_truth) -> tuple[float, float, float]:
    """Token-level F1 (SQuAD style normalisation). Returns (f1, precision, recall)."""
    gts = ground_truth if isinstance(ground_truth, (list, tuple)) else [ground_truth]
    best = (0.0, 0.0, 0.0)
    p = _f1_tokens(prediction or "")
    for g in gts:
        q = _f1_tokens(str(g))
        common = Counter(p) & Counter(q)
        same = sum(common.values())
        if same == 0:
            continue
        prec, rec = same / len(p), same / len(q)
        f1 = 2 * prec * rec / (prec + rec)
        if f1 > best[0]:
            best = (f1, prec, rec)
    return best


def gpqa_reward(response: str, label, metadata: dict | None = None) -> float:
    """Multiple choice: the last standalone option letter (A-J) in the answer part."""
    text = response.split("</think>")[-1]
    m = re.findall(r"(?i)answer\s*(?:is|:)?\s*\(?([A-J])\)?\b", text)
    if not m:
        m = re.findall(r"\b([A-J])\b", text)
    pred = m[-1].upper() if m else None
    gt = str(label).strip().upper()
    if metadata and "correct_letter" in metadata:
        gt = str(metadata["correct_letter"]).upper()
    return 1.0 if pred == gt else 0.0


_IF_CHECKERS = {
    "lowercase": lambda r, kw: r == r.lower(),
    "uppercase": lambda r, kw: r == r.upper(),
    "no_comma": lambda r, kw: "," not in r,
    "min_words": lambda r, kw: len(r.split()) >= int(kw.get("num_words", 0)),
    "max_words": lambda r, kw: len(r.split()) <= int(kw.get("num_words", 1 << 30)),
    "ends_with": lambda r, kw: r.strip().endswith(str(kw.get("end_phrase", ""))),
    "starts_with": lambda r, kw: r.strip().startswith(str(kw.get("start_phrase", ""))),
    "contains": lambda r, kw: all(k in r for k in kw.get("keywords", [])),
    "not_contains": lambda r, kw: not any(k in r for k in kw.get("forbidden_words", [])),
    "num_paragraphs": lambda r, kw: len([p for p in r.split("\n\n") if p.strip()]) == int(kw.get("num_paragraphs", 1)),
    "quotation": lambda r, kw: r.strip().startswith('"') and r.strip().endswith('"'),
    "json_format": lambda r, kw: _is_json(r),
}


def _is_json(r: str) -> bool:
    import json
    try:
        json.loads(r.strip().strip("`").removeprefix("json"))
        return True
    except Exception:
        return False


def ifbench_reward(response: str, label, metadata: dict | None = None) -> float:
    """Fraction of instruction constraints satisfied. `metadata["instructions"]` is a list of
    {"id": checker, "kwargs": {...}} (checkers: lowercase, uppercase, no_comma, min/max_words,
    starts/ends_with, contains, not_contains, num_paragraphs, quotation, json_format)."""
    metadata = metadata or {}
    insts = metadata.get("instructions") or (label if isinstance(label, list) else [])
    if not insts:
        return 0.0
    text = response.split("</think>")[-1].strip()
    ok = 0
    for it in insts:
        cid = it.get("id") if isinstance(it, dict) else str(it)
        kw = it.get("kwargs", {}) if isinstance(it, dict) else {}
        fn = _IF_CHECKERS.get(cid.split(":")[-1] if cid else "")
        if fn is not None and fn(text, kw or {}):
            ok += 1
    return ok / len(insts)


# ----------------------------------------------------------------------------- dispatch
async def remote_rm(args, sample: Sample):
    import aiohttp

    payload = {"prompt": sample.prompt, "response": sample.response, "label": sample.label}
    async with aiohttp.ClientSession() as session:
        async with session.post(args.rm_url, json=payload) as resp:
            resp.raise_for_status()
            return await resp.json()


def rule_based_reward(rm_type: str, response: str, label, metadata: dict | None = None):
    if rm_type.startswith("boxed_"):
        response = last_boxed(response) or ""
        rm_type = rm_type[len("boxed_"):]
    if rm_type == "deepscaler":
        return deepscaler_reward(response, label)
    if rm_type == "dapo":
        return dapo_reward(response, label)
    if rm_type == "math":
        return 1 if grade_answer(response, label) else 0
    if rm_type == "f1":
        return f1_score(response, label)[0]
    if rm_type == "gpqa":
        return gpqa_reward(response, label, metadata)
    if rm_type == "ifbench":
        return ifbench_reward(response, label, metadata)
    if rm_type == "random":
        return random.randint(0, 1)
    if rm_type:
        raise NotImplementedError(f"rule-based RM {rm_type!r} is not implemented")
    raise NotImplementedError("no reward type given (--rm-type or metadata['rm_type'])")


async def async_rm(args, sample: Sample, **kwargs):
    if getattr(args, "custom_rm_path", None):
        return await load_function(args.custom_rm_path)(args, sample, **kwargs)
    md = sample.metadata if isinstance(sample.metadata, dict) else {}
    rm_type = (md.get("rm_type") or getattr(args, "rm_type", None) or "").strip()
    if rm_type == "remote_rm":
        return await remote_rm(args, sample)
    return rule_based_reward(rm_type, sample.response, sample.label, md)


async def batched_async_rm(args, samples: list[Sample], inplace_set_reward_field: bool = False,
                           **kwargs):
    if inplace_set_reward_field:
        rewards = await batched_async_rm(args, samples, **kwargs)
        for s, r in zip(samples, rewards):
            s.reward = r
        return None
    if getattr(args, "custom_rm_path", None):
        return await load_function(args.custom_rm_path)(args, samples, **kwargs)
    return await asyncio.gather(*[async_rm(args, s, **kwargs) for s in samples])
