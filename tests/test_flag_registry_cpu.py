"""Every command-line flag is acted on: read by the code it configures (outside the argument
module), or listed with a reason as needing no action (NO_EFFECT), or rejected when given a
non-default value (UNSUPPORTED)."""
import argparse
import os
import re

import pytest

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _dests():
    from miles_b200.utils import arguments as A

    p = argparse.ArgumentParser()
    for g in A.ALL_GROUPS:
        g(p)
    return sorted({a.dest for a in p._actions if a.dest != "help"})


def _source():
    out = []
    for base in ("miles_b200", "train.py", "train_async.py"):
        path = os.path.join(ROOT, base)
        files = [path] if path.endswith(".py") else [os.path.join(d, f) for d, _, fs in os.walk(path)
                                                      for f in fs if f.endswith(".py")]
        for f in files:
            if f.endswith(os.path.join("utils", "arguments.py")):
                continue
            out.append(open(f).read())
    return "\n".join(out)


def test_every_flag_is_used_documented_or_rejected():
    from miles_b200.utils import arguments as A

    src = _source()
    arg_src = open(os.path.join(ROOT, "miles_b200", "utils", "arguments.py")).read()
    unread = []
    for d in _dests():
        used = re.search(r"\b" + d + r"\b", src) or re.search(r"args\." + d + r"\b", arg_src)
        listed = d in A.NO_EFFECT or d in A.UNSUPPORTED
        if not used and not listed:
            unread.append(d)
        assert not (used and d in A.NO_EFFECT), f"{d} is read but listed as having no effect"
    assert not unread, f"flags parsed but never acted on: {unread}"


def test_unsupported_values_are_rejected():
    from miles_b200.utils.arguments import parse_args

    for argv in (["--rollout-external"], ["--lora-type", "canonical_lora"], ["--qkv-format", "bshd"],
                 ["--use-dynamic-global-batch-size"]):
        with pytest.raises(ValueError, match="not supported"):
            parse_args(["--model-name", "tiny"] + argv)
    parse_args(["--model-name", "tiny", "--qkv-format", "thd"])
