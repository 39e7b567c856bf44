"""OpenAI / Anthropic compatible HTTP server.

Parity: astrai/inference/api/server.py:33-202 (pydantic request schemas,
lazily created FastAPI singleton ``get_app()``, engine built in the lifespan
hook from ``app.state.server_config``, routes ``GET /health``,
``GET /stats``, ``POST /v1/chat/completions``, ``POST /v1/messages``, and
``run_server``). ``app.state.engine`` may be set directly (tests, embedding
the server in another process), in which case the lifespan hook builds
nothing.
"""

from __future__ import annotations

import logging
from contextlib import asynccontextmanager
from pathlib import Path
from typing import Any, Dict, List, Optional, Union

import torch
from pydantic import BaseModel, Field

from astrai_b200.inference.api.anthropic import AnthropicResponseBuilder
from astrai_b200.inference.api.openai import OpenAIResponseBuilder
from astrai_b200.inference.api.protocol import ProtocolHandler

logger = logging.getLogger(__name__)

_app = None


class ChatMessage(BaseModel):
    role: str
    content: Optional[str] = None
    tool_calls: Optional[List[Dict[str, Any]]] = None
    tool_call_id: Optional[str] = None


class FunctionDef(BaseModel):
    name: str
    description: Optional[str] = None
    parameters: Optional[Dict[str, Any]] = None


class ToolDef(BaseModel):
    type: str = "function"
    function: FunctionDef


class ChatCompletionRequest(BaseModel):
    model: str = "astrai"
    messages: List[ChatMessage]
    temperature: Optional[float] = Field(default=1.0, ge=0.0, le=2.0)
    top_p: Optional[float] = Field(default=1.0, ge=0.0, le=1.0)
    top_k: Optional[int] = Field(default=50, ge=0)
    stream: Optional[bool] = False
    stop: Optional[Union[str, List[str]]] = None
    max_tokens: Optional[int] = Field(default=2048, ge=1)
    n: Optional[int] = Field(default=1, ge=1)
    presence_penalty: Optional[float] = Field(default=0.0, ge=-2.0, le=2.0)
    frequency_penalty: Optional[float] = Field(default=0.0, ge=-2.0, le=2.0)
    logit_bias: Optional[Dict[int, float]] = None
    user: Optional[str] = None
    tools: Optional[List[ToolDef]] = None
    tool_choice: Optional[Union[str, Dict[str, Any]]] = "auto"


class AnthropicMessage(BaseModel):
    role: str
    content: Union[str, List[Dict[str, Any]]]


class MessagesRequest(BaseModel):
    model: str = "astrai"
    max_tokens: int = Field(default=1024, ge=1)
    messages: List[AnthropicMessage]
    system: Optional[str] = None
    temperature: Optional[float] = Field(default=1.0, ge=0.0, le=2.0)
    top_p: Optional[float] = Field(default=1.0, ge=0.0, le=1.0)
    top_k: Optional[int] = Field(default=50, ge=0)
    stream: Optional[bool] = False
    stop_sequences: Optional[List[str]] = None


def _create_engine(param_path, device: str = "cuda", dtype: torch.dtype = torch.bfloat16, max_batch_size: int = 16,
                   **engine_kwargs):
    from astrai_b200.inference.engine import InferenceEngine
    from astrai_b200.models import AutoModel
    from astrai_b200.tokenize import AutoTokenizer

    path = Path(param_path)
    if not path.exists():
        raise FileNotFoundError(f"Parameter directory not found: {path}")
    tok = AutoTokenizer.from_pretrained(str(path))
    model = AutoModel.from_pretrained(str(path)).to(device=device, dtype=dtype).eval()
    logger.info("Model loaded on %s (%s)", device, dtype)
    return InferenceEngine(model, tok, max_batch_size=max_batch_size, **engine_kwargs)


def get_app():
    """The FastAPI singleton (created on first call)."""
    global _app
    if _app is None:
        from fastapi import APIRouter, FastAPI, HTTPException

        @asynccontextmanager
        async def lifespan(app):
            cfg = dict(app.state.server_config)
            created = False
            if app.state.engine is None and cfg.get("param_path") is not None:
                app.state.engine = _create_engine(**cfg)
                created = True
            yield
            if created and app.state.engine is not None:
                app.state.engine.shutdown()
                app.state.engine = None

        router = APIRouter()

        def engine():
            eng = _app.state.engine
            if eng is None:
                raise HTTPException(status_code=503, detail="Engine not initialized")
            return eng

        @router.get("/health")
        async def health():
            return {"status": "ok", "model_loaded": _app.state.engine is not None}

        @router.get("/stats")
        async def stats():
            return engine().get_stats()

        @router.post("/v1/chat/completions")
        async def chat_completions(request: ChatCompletionRequest):
            return await ProtocolHandler(request, engine(), OpenAIResponseBuilder()).handle()

        @router.post("/v1/messages")
        async def messages(request: MessagesRequest):
            return await ProtocolHandler(request, engine(), AnthropicResponseBuilder()).handle()

        _app = FastAPI(title="AstrAI-B200 inference server", version="0.1.0", lifespan=lifespan)
        _app.include_router(router)
        _app.state.server_config = {}
        _app.state.engine = None
    return _app


def run_server(param_path, host: str = "0.0.0.0", port: int = 8000, reload: bool = False, device: str = "cuda",
               dtype: torch.dtype = torch.bfloat16, max_batch_size: int = 16, **engine_kwargs) -> None:
    import uvicorn

    app = get_app()
    app.state.server_config = dict(param_path=param_path, device=device, dtype=dtype, max_batch_size=max_batch_size,
                                   **engine_kwargs)
    uvicorn.run(app, host=host, port=port, reload=reload)
