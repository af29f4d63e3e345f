"""OpenAI-compatible HTTP front end on the batched engine
(mu_inference/serving/server.py: same routes, request and response schemas).

Routes: ``GET /health``, ``GET /v1/models``, ``GET /v1/models/{model_id}``,
``POST /v1/completions``, ``POST /v1/chat/completions`` (both with
``stream: true`` as server-sent events ending in ``data: [DONE]``) and
``GET /stats``.  Requests run on :class:`~mu_b200.serving.engine.MuBatchEngine`
(continuous batching, GPU sampling) unless the configuration turns
continuous batching off, as in the reference's ``create_app``.

Prompts are strings when the model directory ships a tokenizer; without one a
completion prompt may be a list of token ids (the OpenAI API's token-array
form) and responses carry the generated ``token_ids`` beside the (then
empty) text.  As in the reference, ``stop``, ``presence_penalty`` and
``frequency_penalty`` are accepted and not applied, and only ``n = 1``.
"""

from __future__ import annotations

import json
import time
import uuid
from typing import Any, AsyncIterator, Dict, List, Optional, Union

from pydantic import BaseModel, Field

from ..core.config import EngineConfig, SamplingParams


# ---- request / response schemas (OpenAI format, reference field names) ---------------
class CompletionRequest(BaseModel):
    model: str
    prompt: Union[str, List[int]]
    max_tokens: int = Field(default=256, ge=1, le=4096)
    temperature: float = Field(default=1.0, ge=0.0, le=2.0)
    top_p: float = Field(default=1.0, ge=0.0, le=1.0)
    top_k: int = Field(default=0, ge=0)
    n: int = Field(default=1, ge=1, le=1)
    stream: bool = False
    stop: Optional[List[str]] = None
    presence_penalty: float = Field(default=0.0, ge=-2.0, le=2.0)
    frequency_penalty: float = Field(default=0.0, ge=-2.0, le=2.0)
    repetition_penalty: float = Field(default=1.0, ge=0.1, le=2.0)
    user: Optional[str] = None


class ChatMessage(BaseModel):
    role: str
    content: str


class ChatCompletionRequest(BaseModel):
    model: str
    messages: List[ChatMessage]
    max_tokens: int = Field(default=256, ge=1, le=4096)
    temperature: float = Field(default=1.0, ge=0.0, le=2.0)
    top_p: float = Field(default=1.0, ge=0.0, le=1.0)
    top_k: int = Field(default=0, ge=0)
    n: int = Field(default=1, ge=1, le=1)
    stream: bool = False
    stop: Optional[List[str]] = None
    presence_penalty: float = Field(default=0.0, ge=-2.0, le=2.0)
    frequency_penalty: float = Field(default=0.0, ge=-2.0, le=2.0)
    repetition_penalty: float = Field(default=1.0, ge=0.1, le=2.0)
    user: Optional[str] = None


class CompletionChoice(BaseModel):
    index: int
    text: str
    logprobs: Optional[Any] = None
    finish_reason: Optional[str] = None
    token_ids: Optional[List[int]] = None


class ChatCompletionChoice(BaseModel):
    index: int
    message: ChatMessage
    finish_reason: Optional[str] = None


class UsageInfo(BaseModel):
    prompt_tokens: int
    completion_tokens: int
    total_tokens: int


class CompletionResponse(BaseModel):
    id: str
    object: str = "text_completion"
    created: int
    model: str
    choices: List[CompletionChoice]
    usage: UsageInfo


class ChatCompletionResponse(BaseModel):
    id: str
    object: str = "chat.completion"
    created: int
    model: str
    choices: List[ChatCompletionChoice]
    usage: UsageInfo


class ModelInfo(BaseModel):
    id: str
    object: str = "model"
    created: int
    owned_by: str = "mu-inference"


class ModelList(BaseModel):
    object: str = "list"
    data: List[ModelInfo]


def _params(req) -> SamplingParams:
    return SamplingParams(max_tokens=req.max_tokens, temperature=req.temperature, top_p=req.top_p,
                          top_k=req.top_k, repetition_penalty=req.repetition_penalty)


def _sse(obj: Dict) -> str:
    return f"data: {json.dumps(obj)}\n\n"


class MuServer:
    """The routes of the reference server over one engine."""

    def __init__(self, engine, model_name: str = "mu-model"):
        from fastapi import FastAPI, HTTPException
        from fastapi.middleware.cors import CORSMiddleware

        self.engine = engine
        self.model_name = model_name
        self.app = FastAPI(title="Mu Inference API (B200)",
                           description="OpenAI-compatible API on the mu_b200 engine",
                           version="1.0.0")
        self.app.add_middleware(CORSMiddleware, allow_origins=["*"], allow_credentials=True,
                                allow_methods=["*"], allow_headers=["*"])
        app = self.app

        @app.get("/health")
        async def health():
            return {"status": "healthy", "model": self.model_name}

        @app.get("/v1/models")
        async def list_models():
            return ModelList(data=[ModelInfo(id=self.model_name, created=int(time.time()))])

        @app.get("/v1/models/{model_id}")
        async def get_model(model_id: str):
            if model_id != self.model_name:
                raise HTTPException(status_code=404, detail="Model not found")
            return ModelInfo(id=self.model_name, created=int(time.time()))

        @app.post("/v1/completions")
        async def create_completion(request: CompletionRequest):
            return await self.completion(request)

        @app.post("/v1/chat/completions")
        async def create_chat_completion(request: ChatCompletionRequest):
            return await self.chat_completion(request)

        @app.get("/stats")
        async def get_stats():
            return self.engine.get_stats()

    # ---- handlers (callable without HTTP) ---------------------------------------------
    async def completion(self, req: CompletionRequest):
        rid = f"cmpl-{uuid.uuid4().hex[:24]}"
        if req.stream:
            from fastapi.responses import StreamingResponse

            return StreamingResponse(self.stream_completion(req, rid),
                                     media_type="text/event-stream")
        out = await self.engine.generate(req.prompt, _params(req), rid)
        return CompletionResponse(
            id=rid, created=int(time.time()), model=self.model_name,
            choices=[CompletionChoice(index=0, text=out.text, finish_reason=out.finish_reason,
                                      token_ids=list(out.token_ids))],
            usage=UsageInfo(**out.usage))

    async def stream_completion(self, req: CompletionRequest, rid: str) -> AsyncIterator[str]:
        async for chunk in self.engine.generate_stream(req.prompt, _params(req), rid):
            choice = {"index": 0, "text": chunk.text, "finish_reason": chunk.finish_reason}
            if chunk.token_id >= 0:
                choice["token_id"] = chunk.token_id
            yield _sse({"id": rid, "object": "text_completion", "created": int(time.time()),
                        "model": self.model_name, "choices": [choice]})
            if chunk.finished:
                yield "data: [DONE]\n\n"
                break

    async def chat_completion(self, req: ChatCompletionRequest):
        rid = f"chatcmpl-{uuid.uuid4().hex[:24]}"
        prompt = self.format_chat_prompt(req.messages)
        if req.stream:
            from fastapi.responses import StreamingResponse

            return StreamingResponse(self.stream_chat(req, rid, prompt),
                                     media_type="text/event-stream")
        out = await self.engine.generate(prompt, _params(req), rid)
        return ChatCompletionResponse(
            id=rid, created=int(time.time()), model=self.model_name,
            choices=[ChatCompletionChoice(index=0,
                                          message=ChatMessage(role="assistant", content=out.text),
                                          finish_reason=out.finish_reason)],
            usage=UsageInfo(**out.usage))

    async def stream_chat(self, req: ChatCompletionRequest, rid: str,
                          prompt: str) -> AsyncIterator[str]:
        async for chunk in self.engine.generate_stream(prompt, _params(req), rid):
            delta = {} if chunk.finished else {"content": chunk.text}
            yield _sse({"id": rid, "object": "chat.completion.chunk", "created": int(time.time()),
                        "model": self.model_name,
                        "choices": [{"index": 0, "delta": delta,
                                     "finish_reason": chunk.finish_reason}]})
            if chunk.finished:
                yield "data: [DONE]\n\n"
                break

    @staticmethod
    def format_chat_prompt(messages: List[ChatMessage]) -> str:
        """Plain role-prefixed transcript ending with the assistant's turn
        (the reference's template, server.py:376-396)."""
        names = {"system": "System", "user": "User", "assistant": "Assistant"}
        parts = [f"{names[m.role]}: {m.content}\n" for m in messages if m.role in names]
        return "".join(parts) + "Assistant:"


def create_app(model_path: str, config: Optional[EngineConfig] = None,
               model_name: Optional[str] = None, use_batch_engine: Optional[bool] = None):
    """FastAPI app serving ``model_path`` (server.py:398-446): MuBatchEngine
    when continuous batching is enabled, else the sequential MuEngine; the
    engine loads at startup and shuts down with the app."""
    from .engine import MuBatchEngine, MuEngine

    config = config or EngineConfig()
    if use_batch_engine is None:
        use_batch_engine = config.scheduler.enable_continuous_batching
    engine = (MuBatchEngine if use_batch_engine else MuEngine)(config=config, model_path=model_path)
    server = MuServer(engine, model_name or str(model_path).rstrip("/").split("/")[-1])

    @server.app.on_event("startup")
    async def startup():
        await engine.initialize(model_path)

    @server.app.on_event("shutdown")
    async def shutdown():
        await engine.shutdown()

    return server.app
