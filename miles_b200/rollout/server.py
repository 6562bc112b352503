"""HTTP server around one rollout engine (the SGLang-server role in disaggregated deployments,
external engines, and the router's workers).

Endpoints (request / response shapes follow the SGLang server the reference drives):
  POST /generate                {input_ids, sampling_params, return_logprob, return_routed_experts}
  GET  /health, /health_generate, /model_info, /get_weight_version
  POST /flush_cache, /abort_request, /pause_generation {mode}, /continue_generation,
       /release_memory_occupation {tags}, /resume_memory_occupation {tags},
       /update_weight_version {new_version}, /start_profile, /stop_profile, /shutdown,
       /load_lora_adapter {lora_path}, /unload_lora_adapter, /weights_checker {action},
       /simulate_crash

Reference: backends/sglang_utils/sglang_engine.py (server launch :55-108, control RPCs
:111-587), sglang.patch (pause modes, weight version, routed experts).
"""
from __future__ import annotations

try:  # module level: FastAPI resolves string annotations against module globals
    from fastapi import Request
except ImportError:  # pragma: no cover
    Request = None

import asyncio
import os
import threading

from miles_b200.engine.engine import RolloutEngine
from miles_b200.rollout.engine_client import LocalEngineClient


def build_app(engine: RolloutEngine, tokenizer=None):
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse

    app = FastAPI()
    client = LocalEngineClient(engine, tokenizer)
    state = {"paused": False, "resume": asyncio.Event(), "profiler": None}
    state["resume"].set()

    @app.post("/generate")
    async def generate(req: Request):
        body = await req.json()
        await state["resume"].wait()
        ids = body.get("input_ids")
        if ids is None and tokenizer is not None:
            ids = tokenizer(body["text"], add_special_tokens=False)["input_ids"]
        out = await client.generate(ids, body.get("sampling_params", {}),
                                    body.get("return_logprob", True),
                                    body.get("return_routed_experts", False))
        re_ = out["meta_info"].get("routed_experts")
        if re_ is not None:
            out["meta_info"]["routed_experts"] = re_.tolist()
        return JSONResponse(out)

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/health_generate")
    async def health_generate():
        await client.generate([1, 2, 3], {"max_new_tokens": 1, "temperature": 0.0})
        return {"status": "ok"}

    @app.get("/model_info")
    async def model_info():
        return {"weight_version": str(engine.model.weight_version),
                "model": engine.cfg.to_dict()}

    @app.get("/get_weight_version")
    async def get_weight_version():
        return {"weight_version": str(engine.model.weight_version)}

    @app.post("/update_weight_version")
    async def update_weight_version(req: Request):
        engine.model.weight_version = int((await req.json())["new_version"])
        return {"success": True}

    @app.post("/flush_cache")
    async def flush_cache():
        return {"success": True}

    @app.post("/abort_request")
    async def abort_request(req: Request):
        client.abort()
        return {"success": True}

    @app.post("/pause_generation")
    async def pause_generation(req: Request):
        mode = (await req.json()).get("mode", "abort")
        state["resume"].clear()
        if mode == "abort":
            client.abort()
        return {"success": True, "mode": mode}

    @app.post("/continue_generation")
    async def continue_generation():
        state["resume"].set()
        return {"success": True}

    @app.post("/release_memory_occupation")
    async def release(req: Request):
        engine.release_memory()
        return {"success": True}

    @app.post("/resume_memory_occupation")
    async def resume(req: Request):
        engine.resume_memory()
        return {"success": True}

    @app.post("/start_profile")
    async def start_profile(req: Request):
        import torch

        body = await req.json() if (await req.body()) else {}
        p = torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU,
                                               torch.profiler.ProfilerActivity.CUDA])
        p.__enter__()
        state["profiler"] = (p, body.get("output_dir", "/tmp/engine_profile"))
        return {"success": True}

    @app.post("/stop_profile")
    async def stop_profile():
        if state["profiler"]:
            p, d = state["profiler"]
            p.__exit__(None, None, None)
            os.makedirs(d, exist_ok=True)
            p.export_chrome_trace(os.path.join(d, "trace.json"))
            state["profiler"] = None
        return {"success": True}

    @app.post("/load_lora_adapter")
    async def load_lora(req: Request):
        """Load adapter tensors saved by `LoRA.save` into the engine's attached adapters."""
        body = await req.json()
        lora = getattr(engine.model, "lora", None)
        if lora is None:
            return JSONResponse({"success": False, "message": "the engine has no LoRA adapters"}, 400)
        lora.load(body["lora_path"])
        return {"success": True}

    @app.post("/unload_lora_adapter")
    async def unload_lora(req: Request):
        """Serve the base weights: the adapters' B matrices are zeroed (reload with
        /load_lora_adapter)."""
        import torch

        lora = getattr(engine.model, "lora", None)
        if lora is None:
            return JSONResponse({"success": False, "message": "the engine has no LoRA adapters"}, 400)
        with torch.no_grad():
            for b in lora.B.values():
                b.zero_()
        return {"success": True}

    @app.post("/weights_checker")
    async def weights_checker(req: Request):
        """action "snapshot": remember a checksum of the weights; "compare": report whether the
        weights still match the snapshot; "checksum": return the current checksum (the bf16 bit
        patterns summed as integers, so equal bits give equal sums)."""
        import torch

        body = await req.json() if (await req.body()) else {}
        flat = engine.model.flat
        csum = int(flat.view(torch.int16).to(torch.int64).sum().item()) if flat.element_size() == 2 else \
            int(flat.view(torch.int32).to(torch.int64).sum().item())
        action = body.get("action", "checksum")
        out = {"success": True, "checksum": csum, "weight_version": str(engine.model.weight_version)}
        if action == "snapshot":
            state["weights_snapshot"] = csum
        elif action == "compare":
            snap = state.get("weights_snapshot")
            out["equal"] = snap is not None and snap == csum
        return out

    @app.post("/simulate_crash")
    async def simulate_crash():
        """Fault injection on the host: the engine is marked dead (health checks fail, generate
        raises) without touching the GPU, so the recovery path can be exercised."""
        engine.dead = True
        return {"success": True}

    @app.post("/shutdown")
    async def shutdown():
        threading.Timer(0.2, lambda: os._exit(0)).start()
        return {"success": True}

    return app


def serve(engine: RolloutEngine, host: str, port: int, tokenizer=None, background: bool = False):
    import uvicorn

    app = build_app(engine, tokenizer)
    cfg = uvicorn.Config(app, host=host, port=port, log_level="warning")
    server = uvicorn.Server(cfg)
    if background:
        t = threading.Thread(target=server.run, daemon=True)
        t.start()
        return server, t
    server.run()
    return server, None
