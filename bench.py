"""Headline benchmark: one colocated GRPO step (rollout + log-probs + policy update) of
Qwen3-30B-A3B (random init, synthetic prompts/rewards) per timed step.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

Workload per GPU (weak scaling): 8 prompts x 8 samples, 512 uniform-random prompt tokens,
responses of uniform 1024..8192 tokens (the length is sampled per response; generation stops
there), temperature 1.0, Bernoulli(0.5) rewards, GRPO advantages, PPO clip 0.2, TIS cap 2.0,
Rollout Routing Replay (routing recorded in rollout, replayed in training), Adam lr 1e-6.
At N GPUs the global batch is N x 64 samples (N x 8 prompts), i.e. the headline workload's
64 prompts x 8 samples at N = 8.

Rollout (default): the reference's partial rollout with over-sampling (--partial-rollout,
--over-sampling-batch-size, here 4x): 32 groups per GPU are in flight, each step trains the first
8 that complete, and the others keep their partial responses for the next step. Every trained sample
is generated to its full sampled length; in steady state each step generates as many tokens as
it trains. `--partial-rollout 0` generates every step's 8 groups to the end instead.

Timing: W untimed warm-up steps, then K steps bracketed by barrier + synchronize, device-timed
with CUDA events; the max over ranks is reported. Inputs are larger than L2 every step (the
model itself is ~61 GB). `e2e` times the same public API call (ColocatedRL.step) on the host
clock, including the host->device copy of the prompts and the device->host read of the result.
A run that would outlast `--time-limit` (wall clock from process start) times fewer steps than
asked and reports both counts (`steps`, `steps_requested`, `stopped_early`).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

T_START = time.perf_counter()


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--prompts-per-gpu", type=int, default=8)
    ap.add_argument("--samples-per-prompt", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--resp-min", type=int, default=1024)
    ap.add_argument("--resp-max", type=int, default=8192)
    ap.add_argument("--max-tokens-per-gpu", type=int, default=16384)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--partial-rollout", type=int, default=1,
                    help="1: reference --partial-rollout with over-sampling (unfinished groups "
                         "continue next step); 0: every step generates its groups to the end")
    ap.add_argument("--over-sampling", type=int, default=4,
                    help="groups in flight per trained group under partial rollout")
    ap.add_argument("--steps-per-sync", type=int, default=8)
    ap.add_argument("--time-limit", type=float, default=None,
                    help="wall-clock seconds (from process start) the whole run must fit in: the "
                         "timed loop ends early, and says so in the JSON line (steps = the steps "
                         "actually timed, steps_requested = K), when one more step would not fit. "
                         "Default 1700 s at one GPU, 820 s per run at several; 0 disables")
    ap.add_argument("--fp8", type=int, default=1,
                    help="1: unified block-scaled fp8 (e4m3, 1x128 activation / 128x128 weight "
                         "scales) forward GEMMs in rollout and training (the headline config); "
                         "0: bf16")
    return ap.parse_args()


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        time.sleep(0.2)
        sm, reasons, smax = [], set(), None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            try:
                sm.append(float(s[1]))
                smax = float(s[2])
                for n, v in zip(names, s[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except Exception:
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


METRIC = "GRPO step s & rollout tok/s at 1/2/4/8 B200 (Qwen3-30B-A3B); weight-sync s"


def reference_arm(args):
    """Runs the unmodified reference through its public entry point when its stack imports;
    otherwise prints the `unavailable` line naming what is missing."""
    here = os.path.dirname(os.path.abspath(__file__))
    ref = os.path.join(here, "baseline", "_ref")
    missing = []
    if os.path.isdir(ref):
        sys.path.insert(0, ref)
        import importlib

        # train.py of the reference imports these through miles.ray / backends
        for mod in ("miles", "ray", "sglang", "megatron.core", "transformer_engine"):
            try:
                importlib.import_module(mod)
            except Exception:  # noqa: BLE001
                missing.append(mod)
        why = ("reference installed in baseline/_ref (pip --no-deps; its dependency 'accelerate' "
               "and the rest of its stack are not in the offline wheelhouse), but its entry point "
               f"cannot run: missing {', '.join(missing)}") if missing else ""
    else:
        why = "baseline/_ref not installed (pip install of the reference failed offline)"
    if int(os.environ.get("RANK", "0")) == 0:
        if why:
            print(json.dumps({"impl": "reference", "unavailable": why, "metric": METRIC}), flush=True)
        else:  # pragma: no cover - not reachable on this image
            print(json.dumps({"impl": "reference", "unavailable": "reference stack imports but the "
                              "8xB200 Ray/SGLang launch is not wired in this bench", "metric": METRIC}),
                  flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    # the KV cache (rollout) and the gradient buffer (training) take turns on the same memory
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    from miles_b200.engine.engine import RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops import _lib
    from miles_b200.ops.rl import PolicyLossCfg
    from miles_b200.trainer.actor import Actor, ActorConfig
    from miles_b200.trainer.grpo import ColocatedRL, RLConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    group = dist.group.WORLD if world > 1 else None

    cfg = preset(args.model)
    model = Transformer(cfg, device=dev, seed=1234)
    if args.fp8:
        model.enable_fp8()
    inflight = args.prompts_per_gpu * (args.over_sampling if args.partial_rollout else 1)
    engine = RolloutEngine(model, max_batch=inflight * args.samples_per_prompt,
                           use_cuda_graph=not args.no_graph, steps_per_sync=args.steps_per_sync,
                           max_pages_per_seq=(args.prompt_len + args.resp_max + 63) // 64 + 1)
    acfg = ActorConfig(lr=1e-6, max_tokens_per_gpu=args.max_tokens_per_gpu,
                       loss=PolicyLossCfg(eps_clip=0.2, eps_clip_high=0.2, use_tis=True,
                                          tis_clip=2.0),
                       use_routing_replay=cfg.is_moe,
                       # old log-probs from the training forward (bitwise those of a separate
                       # no-grad pass; one optimizer step per rollout)
                       old_logp_from_forward=True)
    actor = Actor(model, acfg, dp_group=group)
    rl = ColocatedRL(engine, actor, RLConfig(n_samples_per_prompt=args.samples_per_prompt,
                                             routing_replay=cfg.is_moe, seed=rank,
                                             partial_rollout=bool(args.partial_rollout),
                                             groups_per_step=args.prompts_per_gpu,
                                             over_sampling=args.over_sampling))
    rng = np.random.default_rng(1000 + rank)
    nsamp = args.prompts_per_gpu * args.samples_per_prompt

    def workload():
        """This step's fresh prompt groups (in pinned host memory, copied to the device by the
        step), their sampled response lengths and Bernoulli(0.5) rewards."""
        k = rl.prompts_needed() if args.partial_rollout else args.prompts_per_gpu
        n = k * args.samples_per_prompt
        prompts = torch.from_numpy(rng.integers(0, cfg.vocab_size, (k, args.prompt_len)).astype(np.int32))
        lens = rng.integers(args.resp_min, args.resp_max + 1, n).tolist()
        rewards = (rng.random(n) < 0.5).astype(np.float32).tolist()
        return prompts.pin_memory(), lens, rewards

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def progress(tag, m):
        if rank == 0:
            keys = ("perf/rollout_time", "perf/log_probs_time", "perf/actor_train_time",
                    "perf/step_time", "response_tokens", "rollout/generated_tokens",
                    "rollout/decode_steps", "rollout/preemptions",
                    "train/train_rollout_logprob_abs_diff",
                    "train/train_rollout_logprob_abs_diff_current_weights", "grad_norm")
            print(tag, json.dumps({k: m.get(k) for k in keys}), file=sys.stderr, flush=True)

    for i in range(args.warmup):
        prompts, lens, rewards = workload()
        progress(f"warmup {i}", rl.step(prompts.to(dev, non_blocking=True), lens, rewards))
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    n0 = _lib.launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    tokens = resp = 0
    rollout_s = train_s = lp_s = 0.0
    model.fp8_sync_events.clear()
    t_host0 = time.perf_counter()
    ev0.record()
    h2d = d2h = 0
    limit = args.time_limit if args.time_limit is not None else (1700.0 if world == 1 else 820.0)
    done, slowest, t_prev = 0, 0.0, time.perf_counter()
    for _ in range(args.steps):
        if done and limit > 0:
            # one more step must fit (with 15 % slack on the slowest so far); every rank
            # decides the same way (max over ranks)
            now = time.perf_counter()
            slowest = max(slowest, now - t_prev)
            t_prev = now
            over = torch.tensor([float(now - T_START + 1.15 * slowest > limit)], device=dev)
            if world > 1:
                dist.all_reduce(over, op=dist.ReduceOp.MAX)
            if over.item() > 0:
                break
        prompts, lens, rewards = workload()
        # host -> device: this step's prompt ids from pinned memory; device -> host inside the
        # step: generated tokens / log-probs / routing and the step's metrics
        m = rl.step(prompts.to(dev, non_blocking=True), lens, rewards)
        h2d += prompts.numel() * prompts.element_size()
        d2h += int(m.get("rollout/generated_tokens", 0)) * 8 + 8 * len(m)
        progress("timed", m)
        tokens += m["tokens_total"]
        resp += m["response_tokens"]
        rollout_s += m["perf/rollout_time"]
        lp_s += m["perf/log_probs_time"]
        train_s += m["perf/actor_train_time"]
        done += 1
    ev1.record()
    barrier()
    t_host = time.perf_counter() - t_host0
    clocks = sampler.stop()
    launches = _lib.launch_count() - n0
    ms = ev0.elapsed_time(ev1) / done
    vals = torch.tensor([ms, t_host / done * 1e3, rollout_s, lp_s, train_s,
                         float(tokens), float(resp)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = vals[:5].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = vals[5:].clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        vals = torch.cat([mx, sm])
    sync_s = sum(a.elapsed_time(b) for a, b in model.fp8_sync_events) / 1e3 / done
    ms, host_ms, rollout_s, lp_s, train_s, tokens, resp = vals.tolist()
    step_s = ms / 1e3
    value = tokens / done / step_s
    if rank == 0:
        h2d = h2d // done * world
        d2h = d2h // done * world
        out = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s (GRPO step throughput: prompt+response tokens rolled out and trained per second, whole job)",
            "n_gpus": world, "steps": done, "warmup": args.warmup,
            **({"steps_requested": args.steps,
                "stopped_early": f"time limit {limit:.0f} s (--time-limit): {args.steps} steps "
                                 f"would not fit; {done} timed"} if done < args.steps else {}),
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": ("fp8-block (e4m3 forward GEMMs: 1x128 activation / 128x128 weight scales, "
                      "rollout and training; bf16 backward, attention, LM head, router; fp32 accum)"
                      if args.fp8 else "bf16"),
            "data": "synthetic (uniform-random prompt tokens, Bernoulli(0.5) rewards, random-init weights)",
            "config": {"model": "Qwen3-30B-A3B" if args.model == "qwen3-30b-a3b" else args.model,
                       "global_batch": nsamp * world, "prompts": args.prompts_per_gpu * world,
                       "samples_per_prompt": args.samples_per_prompt, "seq_len": args.prompt_len + args.resp_max,
                       "prompt_len": args.prompt_len, "response_len": [args.resp_min, args.resp_max],
                       "parallelism": f"dp{world}" if world > 1 else "dp1",
                       "routing_replay": cfg.is_moe, "tis_cap": 2.0,
                       "rollout": ({"partial_rollout": True, "over_sampling": args.over_sampling,
                                    "note": "reference --partial-rollout: each step trains the first "
                                            f"{args.prompts_per_gpu} complete groups per GPU; unfinished "
                                            "groups continue next step (TIS corrects the off-policy tokens)"}
                                   if args.partial_rollout else {"partial_rollout": False}),
                       "l2": "inputs larger than L2 (61 GB of weights streamed every step)"},
            "grpo_step_s": step_s,
            "rollout_tok_s": resp / done / (rollout_s / done),
            "rollout_s": rollout_s / done, "log_probs_s": lp_s / done,
            "train_s": train_s / done, "weight_sync_s": sync_s,
            "weight_sync_note": ("colocated engine shares the trainer's parameter buffer; with fp8 the "
                                 "refit is the in-place 128x128 block re-quantisation of every GEMM "
                                 "weight after the optimizer step (device-timed)" if args.fp8 else
                                 "colocated engine shares the trainer's parameter buffer: refit is a "
                                 "weight-version bump"),
            "clocks": clocks,
            "e2e": {"value": tokens / (host_ms / 1e3 * done), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "train_rollout_logprob_abs_diff": rl.last_metrics.get("train/train_rollout_logprob_abs_diff"),
            # over the tokens sampled under the weights being trained (partial rollout resumes
            # samples whose earlier tokens came from older weights): 0.0 = bitwise parity
            "train_rollout_logprob_abs_diff_current_weights":
                rl.last_metrics.get("train/train_rollout_logprob_abs_diff_current_weights"),
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
