"""Class-based rollout functions behind MILES_EXPERIMENTAL_ROLLOUT_REFACTOR=1: the class is
built once from (args, data_source) and called with train / eval inputs (sync or async); a
plain function keeps the legacy call."""
import argparse

from miles_b200.rollout.base_types import (RolloutFnEvalOutput, RolloutFnTrainOutput,
                                           load_rollout_callable, RolloutFnConstructorInput)


class _Rollout:
    built = 0

    def __init__(self, inp):
        _Rollout.built += 1
        self.args, self.ds = inp.args, inp.data_source

    async def __call__(self, inp):
        if inp.evaluation:
            return RolloutFnEvalOutput({"set": {"rewards": [inp.rollout_id]}})
        return RolloutFnTrainOutput([[self.ds, inp.rollout_id]], {"n": self.args.k})


def _legacy(args, rollout_id, data_source, evaluation=False):
    return ("legacy", rollout_id, evaluation)


def test_class_and_legacy_rollout_functions():
    ctor = RolloutFnConstructorInput(argparse.Namespace(k=3), "DS")
    fn = load_rollout_callable(f"{__name__}._Rollout", ctor)
    out = fn(None, 4, None, evaluation=False)
    assert out.samples == [["DS", 4]] and out.metrics == {"n": 3}
    assert fn(None, 5, None, evaluation=True) == {"set": {"rewards": [5]}}
    assert _Rollout.built == 1
    assert load_rollout_callable(f"{__name__}._legacy", ctor)(None, 2, None, evaluation=True) == ("legacy", 2, True)
