"""OpenAI-compatible HTTP frontend and the interactive shell.

Endpoints (same paths and stream formats as the reference,
python/minisgl/server/api_server.py:225-316):

* ``POST /generate`` - raw SSE stream ``data: <text>\\n`` then ``data: [DONE]``;
* ``GET|POST /v1`` - liveness;
* ``POST /v1/chat/completions`` - OpenAI chat completions, streamed as
  ``chat.completion.chunk``-style SSE or returned as one JSON object;
* ``GET /v1/models``.

The frontend hands requests to the tokenizer worker over ZMQ and fans the
incremental replies out to per-request asyncio events. A client that
disconnects mid-stream aborts its request in the scheduler.
"""

from __future__ import annotations

import asyncio
import json
import time
from contextlib import asynccontextmanager
from dataclasses import dataclass, field
from typing import AsyncIterator, Callable, Dict, List, Literal, Optional

from fastapi import Request  # module level: the route signatures' string annotations resolve here
from pydantic import BaseModel, Field

from minisgl.core import SamplingParams
from minisgl.env import ENV
from minisgl.message import AbortMsg, BaseFrontendMsg, BaseTokenizerMsg, BatchFrontendMsg, TokenizeMsg, UserReply
from minisgl.utils import ZmqAsyncPullQueue, ZmqAsyncPushQueue, init_logger

from .args import ServerArgs

logger = init_logger(__name__, "FrontendAPI")


class GenerateRequest(BaseModel):
    prompt: str
    max_tokens: int
    ignore_eos: bool = False


class Message(BaseModel):
    role: Literal["system", "user", "assistant"]
    content: str


class OpenAICompletionRequest(BaseModel):
    model: str
    prompt: Optional[str] = None
    messages: Optional[List[Message]] = None
    max_tokens: int = 16
    temperature: float = 1.0
    top_k: int = -1
    top_p: float = 1.0
    n: int = 1
    stream: bool = False
    stop: List[str] = []
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    ignore_eos: bool = False


class ModelCard(BaseModel):
    id: str
    object: str = "model"
    created: int = Field(default_factory=lambda: int(time.time()))
    owned_by: str = "mini-sglang"
    root: str


class ModelList(BaseModel):
    object: str = "list"
    data: List[ModelCard] = Field(default_factory=list)


def _unwrap(msg: BaseFrontendMsg) -> List[UserReply]:
    if isinstance(msg, BatchFrontendMsg):
        return [m for m in msg.data if isinstance(m, UserReply)]
    assert isinstance(msg, UserReply)
    return [msg]


@dataclass
class FrontendManager:
    config: ServerArgs
    send_tokenizer: ZmqAsyncPushQueue
    recv_tokenizer: ZmqAsyncPullQueue
    uid_counter: int = 0
    listening: bool = False
    ack_map: Dict[int, List[UserReply]] = field(default_factory=dict)
    event_map: Dict[int, asyncio.Event] = field(default_factory=dict)
    prompt_tokens: Dict[int, int] = field(default_factory=dict)

    def new_user(self) -> int:
        uid = self.uid_counter
        self.uid_counter += 1
        self.ack_map[uid] = []
        self.event_map[uid] = asyncio.Event()
        return uid

    async def listen(self) -> None:
        while True:
            for reply in _unwrap(await self.recv_tokenizer.get()):
                if reply.uid in self.ack_map:
                    self.ack_map[reply.uid].append(reply)
                    self.event_map[reply.uid].set()

    async def send_one(self, msg: BaseTokenizerMsg) -> None:
        if not self.listening:
            asyncio.create_task(self.listen())
            self.listening = True
        await self.send_tokenizer.put(msg)

    async def wait_for_ack(self, uid: int) -> AsyncIterator[UserReply]:
        event = self.event_map[uid]
        done = False
        while not done:
            await event.wait()
            event.clear()
            batch, self.ack_map[uid] = self.ack_map[uid], []
            for ack in batch:
                yield ack
                if ack.finished:
                    done = True
                    break
        self.ack_map.pop(uid, None)
        self.event_map.pop(uid, None)

    async def stream_generate(self, uid: int) -> AsyncIterator[bytes]:
        async for ack in self.wait_for_ack(uid):
            yield f"data: {ack.incremental_output}\n".encode()
            if ack.finished:
                break
        yield b"data: [DONE]\n"

    async def stream_chat_completions(self, uid: int) -> AsyncIterator[bytes]:
        first = True
        async for ack in self.wait_for_ack(uid):
            delta: Dict[str, str] = {}
            if first:
                delta["role"], first = "assistant", False
            if ack.incremental_output:
                delta["content"] = ack.incremental_output
            chunk = {"id": f"cmpl-{uid}", "object": "text_completion.chunk",
                     "choices": [{"delta": delta, "index": 0, "finish_reason": None}]}
            yield f"data: {json.dumps(chunk)}\n\n".encode()
            if ack.finished:
                break
        end = {"id": f"cmpl-{uid}", "object": "text_completion.chunk",
               "choices": [{"delta": {}, "index": 0, "finish_reason": "stop"}]}
        yield f"data: {json.dumps(end)}\n\n".encode()
        yield b"data: [DONE]\n\n"

    async def stream_with_cancellation(self, gen: AsyncIterator[bytes], request, uid: int):
        try:
            async for chunk in gen:
                if await request.is_disconnected():
                    logger.info("client disconnected: request %s", uid)
                    raise asyncio.CancelledError
                yield chunk
        except asyncio.CancelledError:
            asyncio.create_task(self.abort_user(uid))
            raise

    async def abort_user(self, uid: int) -> None:
        await asyncio.sleep(0.1)
        self.ack_map.pop(uid, None)
        self.event_map.pop(uid, None)
        logger.warning("aborting request %s", uid)
        await self.send_one(AbortMsg(uid=uid))

    def shutdown(self) -> None:
        self.send_tokenizer.stop()
        self.recv_tokenizer.stop()


_STATE: Optional[FrontendManager] = None


def get_global_state() -> FrontendManager:
    assert _STATE is not None, "the frontend is not initialised"
    return _STATE


def create_app():
    from fastapi import FastAPI
    from fastapi.responses import StreamingResponse

    @asynccontextmanager
    async def lifespan(_app):
        yield
        if _STATE is not None:
            _STATE.shutdown()

    app = FastAPI(title="minisgl API server", version="0.1.0", lifespan=lifespan)

    @app.post("/generate")
    async def generate(req: GenerateRequest, request: Request):
        st = get_global_state()
        uid = st.new_user()
        await st.send_one(TokenizeMsg(uid=uid, text=req.prompt,
                                      sampling_params=SamplingParams(ignore_eos=req.ignore_eos,
                                                                     max_tokens=req.max_tokens)))
        return StreamingResponse(st.stream_with_cancellation(st.stream_generate(uid), request, uid),
                                 media_type="text/event-stream")

    @app.api_route("/v1", methods=["GET", "POST", "HEAD", "OPTIONS"])
    async def v1_root():
        return {"status": "ok"}

    @app.post("/v1/chat/completions")
    async def chat(req: OpenAICompletionRequest, request: Request):
        st = get_global_state()
        if req.messages:
            prompt = [m.model_dump() for m in req.messages]
        elif req.prompt is not None:
            prompt = req.prompt
        else:
            from fastapi import HTTPException

            raise HTTPException(status_code=400, detail="either 'messages' or 'prompt' is required")
        uid = st.new_user()
        await st.send_one(TokenizeMsg(uid=uid, text=prompt, sampling_params=SamplingParams(
            ignore_eos=req.ignore_eos, max_tokens=req.max_tokens, temperature=req.temperature, top_k=req.top_k,
            top_p=req.top_p)))
        if req.stream:
            return StreamingResponse(st.stream_with_cancellation(st.stream_chat_completions(uid), request, uid),
                                     media_type="text/event-stream")
        text, n = "", 0
        async for ack in st.wait_for_ack(uid):
            text += ack.incremental_output
            n += 1
            if ack.finished:
                break
        return {"id": f"chatcmpl-{uid}", "object": "chat.completion", "created": int(time.time()),
                "model": req.model,
                "choices": [{"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": "stop"}],
                "usage": {"prompt_tokens": 0, "completion_tokens": n, "total_tokens": n}}

    @app.get("/v1/models")
    async def models():
        st = get_global_state()
        return ModelList(data=[ModelCard(id=st.config.model_path, root=st.config.model_path)])

    return app


async def shell() -> None:
    """Line-based chat REPL (``/exit`` quits, ``/reset`` clears history)."""
    st = get_global_state()
    history: List[Message] = []
    loop = asyncio.get_running_loop()
    try:
        while True:
            line = (await loop.run_in_executor(None, input, "$ ")).strip()
            if not line:
                continue
            if line == "/exit":
                return
            if line == "/reset":
                history = []
                continue
            if line.startswith("/"):
                print(f"unknown command {line}; use /exit or /reset")
                continue
            history.append(Message(role="user", content=line))
            uid = st.new_user()
            await st.send_one(TokenizeMsg(uid=uid, text=[m.model_dump() for m in history],
                                          sampling_params=SamplingParams(
                                              max_tokens=ENV.SHELL_MAX_TOKENS.value, top_k=ENV.SHELL_TOP_K.value,
                                              top_p=ENV.SHELL_TOP_P.value,
                                              temperature=ENV.SHELL_TEMPERATURE.value)))
            answer = ""
            async for ack in st.wait_for_ack(uid):
                print(ack.incremental_output, end="", flush=True)
                answer += ack.incremental_output
                if ack.finished:
                    break
            print(flush=True)
            history.append(Message(role="assistant", content=answer))
    except (EOFError, KeyboardInterrupt):
        pass
    finally:
        print("Exiting shell...")
        st.shutdown()
        import psutil

        for child in psutil.Process().children(recursive=True):
            child.kill()


def run_api_server(config: ServerArgs, start_backend: Callable[[], object], run_shell: bool = False) -> None:
    global _STATE
    assert _STATE is None, "the frontend is already running"
    _STATE = FrontendManager(
        config=config,
        recv_tokenizer=ZmqAsyncPullQueue(config.zmq_frontend_addr, create=True, decoder=BaseFrontendMsg.decoder),
        send_tokenizer=ZmqAsyncPushQueue(config.zmq_tokenizer_addr, create=config.frontend_create_tokenizer_link,
                                         encoder=BaseTokenizerMsg.encoder),
    )
    start_backend()
    logger.info(f"API server is ready on {config.server_host}:{config.server_port}")
    if run_shell:
        asyncio.run(shell())
    else:
        import uvicorn

        uvicorn.run(create_app(), host=config.server_host, port=config.server_port)
