"""HTTP front end (the reference ships only a stub that exits,
``kunserve/api_server/kunserve_api_server.py:14-25``).

    python -m kunserve_b200.api_server.server --model tiny-llama --dtype fp32 --cpu --port 8000

Endpoints: ``POST /generate`` (``prompt`` or ``prompt_token_ids``,
``max_tokens``, ``temperature``, ``top_p``, ``top_k``, ``ignore_eos``) returns
the generated ids (and text with a tokenizer) plus TTFT/TPOT; ``GET /health``;
``GET /metrics`` returns the server's epoch counters as JSON.
"""
import argparse
from typing import List, Optional

from fastapi import FastAPI, HTTPException
from pydantic import BaseModel

from ..request import SamplingParams


class GenerateRequest(BaseModel):
    prompt: Optional[str] = None
    prompt_token_ids: Optional[List[int]] = None
    max_tokens: int = 16
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = -1
    ignore_eos: bool = False


def build_app(llm_factory) -> FastAPI:
    """``llm_factory`` is an async callable returning a started ``AsyncLLM``."""
    app = FastAPI(title="kunserve_b200")
    state = {}

    @app.on_event("startup")
    async def _start():
        state["llm"] = await llm_factory()

    @app.on_event("shutdown")
    async def _stop():
        if "llm" in state:
            await state["llm"].terminate()

    @app.get("/health")
    async def health():
        return {"ok": "llm" in state}

    @app.get("/metrics")
    async def metrics():
        return state["llm"].report_server_metrics()

    @app.post("/generate")
    async def generate(req: GenerateRequest):
        if req.prompt is None and req.prompt_token_ids is None:
            raise HTTPException(400, "need prompt or prompt_token_ids")
        try:
            sp = SamplingParams(temperature=req.temperature, top_p=req.top_p, top_k=req.top_k,
                                max_tokens=req.max_tokens, ignore_eos=req.ignore_eos)
        except ValueError as e:
            raise HTTPException(400, str(e))
        out = await state["llm"].generate(prompt=req.prompt, prompt_token_ids=req.prompt_token_ids,
                                          sampling_params=sp)
        m = out["metrics"]
        return {"request_id": out["request_id"], "token_ids": out["outputs"], "text": out["text"],
                "prompt_len": out["prompt_len"], "ttft_s": m.ttft, "tpot_s": m.tbt}

    return app


def main(argv=None):
    import uvicorn

    from ..config import ModelConfig, add_cli_args, get_cli_args
    from ..llm import AsyncLLM

    p = add_cli_args(argparse.ArgumentParser("kunserve_b200 api server"))
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--cpu", action="store_true")
    a = p.parse_args(argv)
    cfg = get_cli_args(a)
    mc = ModelConfig(cfg.bench_config.model or "tiny-llama", dtype=cfg.engine_config.dtype)

    async def factory():
        kw = {"backend": "torch", "devices": ["cpu"]} if a.cpu else {}
        return await AsyncLLM.create(cfg, model_config=mc, num_gpu_blocks=cfg.bench_config.num_gpu_blocks, **kw)

    uvicorn.run(build_app(factory), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
