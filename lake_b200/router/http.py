"""HTTP front of the router (aiohttp): POST /v1/chat/completions, GET /healthz,
GET /metrics (Prometheus text).

The chat response follows the OpenAI chat.completion shape plus a ``lake``
object (reused_blocks, prefill_blocks, mode). Upstream failures map to HTTP
codes without leaking backend detail: INVALID_ARGUMENT -> 400, UNAVAILABLE /
DEADLINE_EXCEEDED / RESOURCE_EXHAUSTED -> 503, anything else -> 502.

Reference parity: go/router/server.go:193-421.
"""
from __future__ import annotations

import json
import logging
import os
import time

from aiohttp import web

from .server import MAX_BODY, Router, RouterConfig, RouterError
from .tokenizer import Tokenizer

LOG = logging.getLogger("lake_b200.router")


def make_app(router: Router, tokenizer: Tokenizer | None = None) -> web.Application:
    tokenizer = tokenizer or Tokenizer.from_env()

    async def healthz(_req):
        return web.Response(text="ok")

    async def metrics(_req):
        return web.Response(text=router.metrics_text(), content_type="text/plain")

    async def chat(req: web.Request):
        if req.content_length is not None and req.content_length > MAX_BODY:
            return web.Response(status=413, text="request body too large")
        try:
            body = await req.read()
        except Exception:
            return web.Response(status=413, text="request body too large")
        if len(body) > MAX_BODY:
            return web.Response(status=413, text="request body too large")
        try:
            data = json.loads(body)
            if not isinstance(data, dict):
                raise ValueError
        except ValueError:
            return web.Response(status=400, text="invalid JSON request")
        try:
            tokens = tokenizer.encode_request(data)
        except Exception as e:  # a message the chat template cannot render; the detail stays in the log
            LOG.info("cannot tokenize request: %s", e)
            return web.Response(status=400, text="cannot tokenize request")
        max_new = int(data.get("max_tokens") or 0) or 4
        model = data.get("model") or "mock-llm"
        session = req.headers.get("X-Lake-Session-Id", "").encode()
        try:
            out = await router.generate(model, tokens, max_new, int(data.get("priority") or 0), session)
        except RouterError as e:
            return web.Response(status=e.status, text=str(e))
        return web.json_response({
            "id": "chatcmpl-" + out["request_id"][:8], "object": "chat.completion", "created": int(time.time()),
            "model": model,
            "choices": [{"index": 0, "message": {"role": "assistant", "content": tokenizer.decode(out["output_tokens"])},
                         "finish_reason": "stop"}],
            "lake": {"reused_blocks": out["reused_blocks"], "prefill_blocks": out["prefill_blocks"],
                     "mode": out["mode"], "node": out["node"]},
        })

    app = web.Application(client_max_size=MAX_BODY + 1024)
    app.router.add_get("/healthz", healthz)
    app.router.add_get("/metrics", metrics)
    app.router.add_post("/v1/chat/completions", chat)

    async def on_start(_app):
        await router.start()

    async def on_stop(_app):
        await router.close()

    app.on_startup.append(on_start)
    app.on_cleanup.append(on_stop)
    return app


def main() -> None:
    logging.basicConfig(level=os.environ.get("LAKE_LOG", "INFO"))
    host, _, port = os.environ.get("LAKE_HTTP_ADDR", "0.0.0.0:8080").rpartition(":")
    web.run_app(make_app(Router(RouterConfig.from_env())), host=host or "0.0.0.0", port=int(port))


if __name__ == "__main__":
    main()
