"""Engine server control RPCs: LoRA adapter load / unload, the weight checker (snapshot /
compare / checksum) and the host-side simulated crash that the health checks then report."""
import torch
from fastapi.testclient import TestClient

from miles_b200.engine.engine import RolloutEngine
from miles_b200.models.config import preset
from miles_b200.models.lora import LoRA
from miles_b200.models.transformer import Transformer
from miles_b200.rollout.server import build_app


def test_engine_server_rpcs(tmp_path):
    m = Transformer(preset("tiny"), device="cpu", dtype=torch.float32, seed=0)
    m.lora = LoRA(m, 4, 8, ["q_proj", "o_proj"], 0.0, seed=0)
    with torch.no_grad():
        for b in m.lora.B.values():
            b.normal_()
    m.lora.save(str(tmp_path / "a.pt"))
    eng = RolloutEngine(m, max_batch=2, num_pages=32, max_pages_per_seq=4, use_cuda_graph=False)
    app = TestClient(build_app(eng))
    gen = {"input_ids": [1, 2, 3, 4], "sampling_params": {"max_new_tokens": 3, "temperature": 0.0}}
    with_lora = app.post("/generate", json=gen).json()["output_ids"]
    assert app.post("/unload_lora_adapter").json()["success"]
    assert all(float(b.abs().sum()) == 0 for b in m.lora.B.values())
    assert app.post("/load_lora_adapter", json={"lora_path": str(tmp_path / "a.pt")}).json()["success"]
    assert app.post("/generate", json=gen).json()["output_ids"] == with_lora
    snap = app.post("/weights_checker", json={"action": "snapshot"}).json()
    assert app.post("/weights_checker", json={"action": "compare"}).json()["equal"]
    with torch.no_grad():
        m.flat[0] += 1.0
    cmp = app.post("/weights_checker", json={"action": "compare"}).json()
    assert not cmp["equal"] and cmp["checksum"] != snap["checksum"]
    assert app.post("/simulate_crash").json()["success"]
    assert not eng.health_check()
