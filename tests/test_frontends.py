"""Public entry points on CPU: the HTTP server and the serving driver."""
import asyncio
import os
import sys

from kunserve_b200.config import KunServeConfig, ModelConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _factory():
    from kunserve_b200.llm import AsyncLLM
    cfg = KunServeConfig()
    cfg.engine_config.block_size = 16

    async def make():
        return await AsyncLLM.create(cfg, model_config=ModelConfig("tiny-llama", dtype="fp32"), backend="torch",
                                     devices=["cpu"], num_gpu_blocks=32)
    return make


def test_http_generate():
    from fastapi.testclient import TestClient
    from kunserve_b200.api_server.server import build_app
    with TestClient(build_app(_factory())) as c:
        assert c.get("/health").json()["ok"]
        r = c.post("/generate", json={"prompt_token_ids": [1, 2, 3, 4], "max_tokens": 5, "ignore_eos": True})
        assert r.status_code == 200 and len(r.json()["token_ids"]) == 5
        assert c.post("/generate", json={"max_tokens": 5}).status_code == 400
        assert "tokens" in c.get("/metrics").json()


def test_serve_bench_cpu(tmp_path):
    sys.path.insert(0, os.path.join(ROOT, "evaluation"))
    import serve_bench
    s = serve_bench.main(["--model", "tiny-llama", "--dtype", "fp32", "--cpu", "--nlimit", "8", "--qps", "20",
                          "--block-size", "16", "--num-gpu-blocks", "64", "--max-model-len", "256",
                          "--log-path", str(tmp_path), "--log-name", "run"])
    assert s["num_requests"] == 8
    assert os.path.exists(tmp_path / "run.csv") and os.path.exists(tmp_path / "run.parquet")


def test_dataset_builder(tmp_path):
    sys.path.insert(0, os.path.join(ROOT, "evaluation", "data"))
    import build_dataset
    import pandas as pd
    out = tmp_path / "d.parquet"
    build_dataset.main(["--out", str(out), "--n", "20"])
    df = pd.read_parquet(out)
    assert list(df.columns) == ["prompt", "prompt_len", "response_len"] and len(df) == 20
