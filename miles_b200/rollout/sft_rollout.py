"""SFT "rollout": turns chat-message samples into training samples with multi-turn loss masks
(no generation). Use with --loss-type sft_loss and
--rollout-function-path miles_b200.rollout.sft_rollout.generate_rollout.

Each sample's prompt is a list of {"role", "content"} messages. Tokens are the rendered
conversation; the "response" starts at the first trained token (the first assistant turn),
and the loss mask marks the assistant turns inside it.

Reference: miles/rollout/sft_rollout.py:17-66.
"""
from __future__ import annotations

from miles_b200.rollout.default import GenerateState, RolloutFnTrainOutput
from miles_b200.utils.mask_utils import multi_turn_loss_mask
from miles_b200.utils.types import Sample


def build_sft_sample(tokenizer, sample: Sample) -> Sample:
    ids, mask = multi_turn_loss_mask(tokenizer, sample.prompt, sample.metadata.get("tools"))
    if 1 not in mask:
        raise ValueError(f"sample {sample.index} has no assistant turn to train on")
    start = mask.index(1)
    sample.tokens = ids
    sample.response_length = len(ids) - start
    sample.loss_mask = mask[start:]
    sample.reward = 0.0
    sample.status = Sample.Status.COMPLETED
    return sample


def generate_rollout(args, rollout_id: int, data_source, evaluation: bool = False):
    if evaluation:
        raise ValueError("SFT rollout has no evaluation mode")
    tok = GenerateState.get(args).tokenizer
    groups = data_source.get_samples(args.rollout_batch_size)
    out = [[build_sft_sample(tok, s) for s in g] for g in groups]
    return RolloutFnTrainOutput(out, {"sft/num_samples": sum(len(g) for g in out)})
