"""Agentic generate through the session server (CPU, tiny model): a scripted agent makes two
chat calls with a tool message in between; the trajectory comes back with the generated tokens
under loss mask 1 (the tool tokens 0) and the engine's log-probs; multi-sample mode splits it
per assistant turn; a role outside --tito-allowed-append-roles is refused."""
import asyncio
import os
import types

import pytest

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


class _Tok:
    """Character-level tokenizer with a prefix-stable chat template."""

    def encode(self, text, add_special_tokens=False):
        return [ord(c) % 256 for c in text]

    def decode(self, ids):
        return "".join(chr(65 + (i % 26)) for i in ids)

    def apply_chat_template(self, messages, tools=None, tokenize=False, add_generation_prompt=False, **kw):
        text = "".join(f"<{m['role']}>{m['content']}</>" for m in messages)
        if add_generation_prompt:
            text += "<assistant>"
        return self.encode(text) if tokenize else text


async def _agent(base_url, prompt, request_kwargs, metadata, **kw):
    import aiohttp

    msgs = [{"role": "user", "content": "hi"}]
    async with aiohttp.ClientSession() as s:
        for turn in range(2):
            async with s.post(f"{base_url}/chat/completions",
                              json={"messages": msgs, "max_tokens": 5, "seed": turn}) as r:
                out = await r.json()
            msgs.append(out["choices"][0]["message"])
            msgs.append({"role": "tool", "content": f"result{turn}"})
        msgs.pop()
    return {"agent_turns": 2}


def test_agentic_generate_with_session_server():
    import torch

    from miles_b200.engine.engine import RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.rollout import agentic
    from miles_b200.rollout.engine_client import LocalEngineClient
    from miles_b200.rollout.session import launch_session_server
    from miles_b200.utils.types import Sample

    m = Transformer(preset("tiny"), device="cpu", dtype=torch.float32, seed=0)
    eng = RolloutEngine(m, max_batch=4, num_pages=64, use_cuda_graph=False)
    args = types.SimpleNamespace(session_server_ip="127.0.0.1", session_server_port=None,
                                 rollout_max_response_len=16, tito_allowed_append_roles=["tool", "user"],
                                 tito_model=None, custom_agent_function_path="tests.test_agentic_cpu._agent",
                                 generate_multi_samples=False, max_seq_len=None)
    tok = _Tok()
    launch_session_server(args, tok, LocalEngineClient(eng, tok))
    import time

    time.sleep(1.0)
    s = asyncio.run(agentic.generate(args, Sample(prompt="hi", index=0), {"max_new_tokens": 5}))
    assert s.status == Sample.Status.COMPLETED and s.metadata["agent_turns"] == 2
    assert sum(s.loss_mask) == 10 and 0 in s.loss_mask          # 2 x 5 generated, tool tokens masked
    assert len(s.rollout_log_probs) == s.response_length == len(s.loss_mask)
    args.generate_multi_samples = True
    ss = asyncio.run(agentic.generate(args, Sample(prompt="hi", index=1), {"max_new_tokens": 5}))
    assert len(ss) == 2 and all(x.response_length == 5 for x in ss)
    assert ss[1].tokens[: len(ss[0].tokens)] == ss[0].tokens


def test_append_role_policy():
    from miles_b200.rollout.session import Session, SessionError

    tok = _Tok()
    sess = Session()
    ids, mask, lps = sess.prepare(tok, [{"role": "user", "content": "a"}], allowed_roles={"tool"})
    sess.commit([{"role": "user", "content": "a"}], {"role": "assistant", "content": "b"}, ids, mask, lps,
                [1, 2], [-0.1, -0.2])
    with pytest.raises(SessionError, match="not allowed"):
        sess.prepare(tok, sess.messages + [{"role": "system", "content": "x"}], allowed_roles={"tool"})
    sess.prepare(tok, sess.messages + [{"role": "tool", "content": "x"}], allowed_roles={"tool"})
