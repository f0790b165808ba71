"""1P1D proxy: one prefill per paired execution, store-completion gating, decode forwarding.

Behavioural parity with the reference's experiments/progressive_pd_proxy.py:
  * request validation of the proxy-owned ``sparsecache_*`` fields (mode
    baseline|progressive, visibility continuous|fixed_s1, max draft tokens,
    start fraction in (0, 1), request-scoped chunk priority, paired prefill
    group) and greedy-only requests (:137-214);
  * the prefill request is the client request with ``max_tokens=1``,
    non-streaming, ``return_token_ids``; the seed token comes from
    ``choices[0].token_ids[0]`` (:123-135);
  * the decode request carries proxy-owned ``kv_transfer_params``
    (``require_full_remote_kv``; the progressive draft settings with the
    exact producer seed, or ``producer_seed_token_id`` for the baseline);
  * the decode is forwarded only after the prefill worker reported store
    completion on the telemetry endpoint (:217-242, :431-435);
  * a prefill group is prefilled once and its seed reused by every arm of a
    paired execution, with a fingerprint check that refuses a group reused
    for another prompt (409) (:267-330);
  * responses carry ``X-SparseCache-*`` headers and ``Server-Timing``
    (prefill, store_wait, decode) (:331-413).
Requests are serialised (one in flight), as latency cells need.

The HTTP clients of the prefill and decode workers are injectable
(``client_factory``), which lets tests run the whole chain in process.
"""
from __future__ import annotations

import argparse
import asyncio
import hashlib
import json
import logging
import threading
import time
import uuid
from dataclasses import dataclass
from typing import Any, Callable

from fastapi import Request  # module level: FastAPI resolves handler annotations here

LOG = logging.getLogger("sparsecache.proxy")


@dataclass(frozen=True)
class ProxyConfig:
    host: str = "127.0.0.1"
    port: int = 8000
    telemetry_port: int = 5768
    prefiller_url: str = "http://127.0.0.1:8100"
    decoder_url: str = "http://127.0.0.1:8200"
    default_mode: str = "progressive"
    default_visibility_mode: str = "continuous"
    max_draft_tokens: int = 8
    start_fraction: float = 0.05
    require_greedy: bool = True


def build_config(args: argparse.Namespace) -> ProxyConfig:
    if args.max_draft_tokens < 1:
        raise ValueError("max_draft_tokens must be positive")
    if not 0.0 < args.start_fraction < 1.0:
        raise ValueError("start_fraction must lie in (0, 1)")
    return ProxyConfig(args.host, args.port, args.telemetry_port, args.prefiller_url.rstrip("/"),
                       args.decoder_url.rstrip("/"), args.default_mode, args.default_visibility_mode,
                       args.max_draft_tokens, args.start_fraction, args.require_greedy)


def prefill_fingerprint(endpoint: str, payload: dict[str, Any]) -> str:
    blob = json.dumps({"endpoint": endpoint, "payload": payload}, sort_keys=True, separators=(",", ":"),
                      ensure_ascii=False).encode()
    return hashlib.sha256(blob).hexdigest()


def extract_seed_token(response: dict[str, Any]) -> int:
    try:
        seed = response["choices"][0]["token_ids"][0]
    except (KeyError, IndexError, TypeError) as exc:
        raise RuntimeError("prefiller response did not contain choices[0].token_ids[0]; "
                           "the prefiller must support return_token_ids") from exc
    if not isinstance(seed, int) or isinstance(seed, bool):
        raise TypeError("prefiller seed token ID is not an integer")
    return seed


def _is_int(x) -> bool:
    return isinstance(x, int) and not isinstance(x, bool)


def prepare_requests(request: dict[str, Any], config: ProxyConfig, seed_token_id: int | None):
    """Split a client request into (prefill payload, decode payload, mode)."""
    payload = dict(request)
    mode = payload.pop("sparsecache_mode", config.default_mode)
    visibility = payload.pop("sparsecache_visibility_mode", config.default_visibility_mode)
    gamma = payload.pop("sparsecache_max_draft_tokens", config.max_draft_tokens)
    start = payload.pop("sparsecache_start_fraction", config.start_fraction)
    priority = payload.pop("sparsecache_priority_chunks", None)
    group = payload.pop("sparsecache_prefill_group", None)
    if mode not in ("baseline", "progressive"):
        raise ValueError("sparsecache_mode must be baseline or progressive")
    if visibility not in ("continuous", "fixed_s1"):
        raise ValueError("sparsecache_visibility_mode must be continuous or fixed_s1")
    if not _is_int(gamma) or gamma < 1:
        raise ValueError("sparsecache_max_draft_tokens must be a positive integer")
    if isinstance(start, bool) or not isinstance(start, (int, float)) or not 0.0 < float(start) < 1.0:
        raise ValueError("sparsecache_start_fraction must lie in (0, 1)")
    if priority is not None and (not isinstance(priority, list) or not priority
                                 or any(not _is_int(c) or c < 0 for c in priority)
                                 or len(priority) != len(set(priority))):
        raise ValueError("sparsecache_priority_chunks must be unique non-negative integers")
    if group is not None and (not isinstance(group, str) or not group.strip()):
        raise ValueError("sparsecache_prefill_group must be a non-empty string")
    if config.require_greedy and float(payload.get("temperature", 1.0)) != 0.0:
        raise ValueError("the correctness gate requires temperature=0")
    pre = dict(payload)
    pre["max_tokens"] = 1
    if "max_completion_tokens" in pre:
        pre["max_completion_tokens"] = 1
    pre["stream"] = False
    pre.pop("stream_options", None)
    pre["return_token_ids"] = True
    dec = dict(payload)
    params = dict(dec.get("kv_transfer_params") or {})
    if "require_full_remote_kv" in params:
        raise ValueError("kv_transfer_params.require_full_remote_kv is proxy-owned")
    params["require_full_remote_kv"] = True
    if mode == "progressive":
        if seed_token_id is None:
            raise ValueError("progressive mode requires the exact prefiller seed")
        if "progressive_sparse_draft" in params:
            raise ValueError("kv_transfer_params.progressive_sparse_draft is proxy-owned")
        params["progressive_sparse_draft"] = {"seed_token_id": seed_token_id, "max_draft_tokens": gamma,
                                              "start_fraction": float(start), "visibility_mode": visibility}
        if priority is not None:
            params["progressive_priority_chunks"] = priority
        dec["kv_transfer_params"] = params
    elif seed_token_id is not None:
        if "producer_seed_token_id" in params:
            raise ValueError("kv_transfer_params.producer_seed_token_id is proxy-owned")
        params["producer_seed_token_id"] = seed_token_id
        dec["kv_transfer_params"] = params
    return pre, dec, mode


@dataclass(frozen=True)
class PrefillCacheEntry:
    fingerprint: str
    seed_token_id: int


class Proxy:
    """The proxy's state and its two FastAPI apps (API and telemetry)."""

    def __init__(self, config: ProxyConfig, *, client_factory: Callable[[str], Any] | None = None,
                 store_timeout_s: float = 600.0) -> None:
        self.config = config
        self.client_factory = client_factory
        self.store_timeout_s = store_timeout_s
        self.pending: dict[str, asyncio.Event] = {}
        self.pending_lock = threading.Lock()
        self.loop: asyncio.AbstractEventLoop | None = None
        self.request_lock: asyncio.Lock | None = None
        self.prefill_cache: dict[str, PrefillCacheEntry] = {}
        self.app = self._make_app()
        self.telemetry_app = self._make_telemetry_app()

    def _client(self, base_url: str):
        if self.client_factory is not None:
            return self.client_factory(base_url)
        import httpx

        # loopback services: never route 127.0.0.1 through an inherited proxy
        return httpx.AsyncClient(base_url=base_url, timeout=None, trust_env=False)

    def notify(self, raw_request_id: str) -> bool:
        """Telemetry callback: the prefill worker stored the KV of ``raw_request_id``."""
        with self.pending_lock:
            rid = next((c for c in self.pending if raw_request_id == c
                        or raw_request_id.startswith((f"chatcmpl-{c}", f"cmpl-{c}"))), None)
            ev = self.pending.get(rid) if rid is not None else None
        if ev is None or self.loop is None:
            return False
        self.loop.call_soon_threadsafe(ev.set)
        return True

    def _make_telemetry_app(self):
        from fastapi import FastAPI

        app = FastAPI()

        @app.post("/api/v1/telemetry")
        async def telemetry(request: Request):
            body = await request.json()
            ids = body.get("request_ids_set", [])
            return {"status": "ok", "notified": sum(self.notify(str(i)) for i in ids), "total": len(ids)}

        return app

    def _make_app(self):
        from contextlib import asynccontextmanager

        from fastapi import FastAPI, HTTPException
        from fastapi.responses import JSONResponse, StreamingResponse
        from starlette.background import BackgroundTask

        proxy = self

        @asynccontextmanager
        async def lifespan(app):
            proxy.loop = asyncio.get_running_loop()
            proxy.request_lock = asyncio.Lock()
            app.state.prefiller = proxy._client(proxy.config.prefiller_url)
            app.state.decoder = proxy._client(proxy.config.decoder_url)
            yield
            await app.state.prefiller.aclose()
            await app.state.decoder.aclose()

        app = FastAPI(lifespan=lifespan)

        def headers(rid: str) -> dict[str, str]:
            return {"Content-Type": "application/json", "X-Request-Id": rid}

        async def forward(endpoint: str, request: Request):
            if proxy.loop is None:  # lifespan not run (e.g. an ASGI transport without it)
                proxy.loop = asyncio.get_running_loop()
                proxy.request_lock = asyncio.Lock()
                app.state.prefiller = proxy._client(proxy.config.prefiller_url)
                app.state.decoder = proxy._client(proxy.config.decoder_url)
            await proxy.request_lock.acquire()
            release_later = False
            try:
                received = time.perf_counter()
                try:
                    body = await request.json()
                    if not isinstance(body, dict):
                        raise TypeError("request body must be a JSON object")
                    pre_payload, _, mode = prepare_requests(body, proxy.config, seed_token_id=0)
                    group = body.get("sparsecache_prefill_group")
                except (TypeError, ValueError) as exc:
                    raise HTTPException(status_code=400, detail=str(exc)) from exc
                rid = uuid.uuid4().hex[:16]
                fp = prefill_fingerprint(endpoint, pre_payload)
                cached = proxy.prefill_cache.get(group) if group is not None else None
                if cached is not None and cached.fingerprint != fp:
                    raise HTTPException(status_code=409,
                                        detail="sparsecache_prefill_group was reused for a different prompt")
                t_pre = time.perf_counter()
                if cached is not None:
                    seed, t_resp, t_store, reused = cached.seed_token_id, t_pre, t_pre, True
                else:
                    ev = asyncio.Event()
                    with proxy.pending_lock:
                        proxy.pending[rid] = ev
                    try:
                        resp = await app.state.prefiller.post(endpoint, json=pre_payload, headers=headers(rid))
                        resp.raise_for_status()
                        t_resp = time.perf_counter()
                        seed = extract_seed_token(resp.json())
                        await asyncio.wait_for(ev.wait(), timeout=proxy.store_timeout_s)
                        t_store = time.perf_counter()
                    except (asyncio.TimeoutError, RuntimeError, TypeError, Exception) as exc:  # noqa: BLE001
                        if isinstance(exc, HTTPException):
                            raise
                        raise HTTPException(status_code=502, detail=f"prefill failed: {exc!r}") from exc
                    finally:
                        with proxy.pending_lock:
                            proxy.pending.pop(rid, None)
                    reused = False
                    if group is not None:
                        proxy.prefill_cache[group] = PrefillCacheEntry(fp, seed)
                try:
                    _, dec_payload, mode = prepare_requests(body, proxy.config, seed_token_id=seed)
                except ValueError as exc:
                    raise HTTPException(status_code=400, detail=str(exc)) from exc
                t_dec = time.perf_counter()
                common = {
                    "X-SparseCache-Mode": mode, "X-SparseCache-Request-Id": rid,
                    "X-SparseCache-Seed-Token": str(seed), "X-SparseCache-Prefill-Reused": str(reused).lower(),
                    "X-SparseCache-Prefill-Group": group or "",
                    "Server-Timing": (f"prefill;dur={(t_resp - t_pre) * 1000:.3f}, "
                                      f"store_wait;dur={(t_store - t_resp) * 1000:.3f}"),
                }
                LOG.info("request=%s mode=%s reused=%s prefill_ms=%.3f", rid, mode, reused, (t_resp - t_pre) * 1e3)
                if dec_payload.get("stream", False):
                    async def stream():
                        async with app.state.decoder.stream("POST", endpoint, json=dec_payload,
                                                            headers=headers(rid)) as r:
                            r.raise_for_status()
                            async for chunk in r.aiter_bytes():
                                yield chunk

                    release_later = True
                    return StreamingResponse(stream(), media_type="text/event-stream", headers=common,
                                             background=BackgroundTask(proxy.request_lock.release))
                try:
                    r = await app.state.decoder.post(endpoint, json=dec_payload, headers=headers(rid))
                    r.raise_for_status()
                except Exception as exc:  # noqa: BLE001
                    raise HTTPException(status_code=502, detail=str(exc)) from exc
                done = time.perf_counter()
                common["Server-Timing"] += f", decode;dur={(done - t_dec) * 1000:.3f}"
                LOG.info("request=%s total_ms=%.3f", rid, (done - received) * 1e3)
                return JSONResponse(r.json(), status_code=r.status_code, headers=common)
            finally:
                if not release_later:
                    proxy.request_lock.release()

        @app.post("/v1/completions")
        async def completions(request: Request):
            return await forward("/v1/completions", request)

        @app.post("/v1/chat/completions")
        async def chat_completions(request: Request):
            return await forward("/v1/chat/completions", request)

        @app.get("/v1/models")
        async def models():
            if getattr(app.state, "prefiller", None) is None:
                app.state.prefiller = proxy._client(proxy.config.prefiller_url)
            r = await app.state.prefiller.get("/v1/models")
            return JSONResponse(r.json(), status_code=r.status_code)

        @app.get("/health")
        async def health():
            return {"status": "ok"}

        return app


def main(argv=None) -> None:
    import uvicorn

    p = argparse.ArgumentParser()
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--telemetry-port", type=int, default=5768)
    p.add_argument("--prefiller-url", default="http://127.0.0.1:8100")
    p.add_argument("--decoder-url", default="http://127.0.0.1:8200")
    p.add_argument("--default-mode", choices=("baseline", "progressive"), default="progressive")
    p.add_argument("--default-visibility-mode", choices=("continuous", "fixed_s1"), default="continuous")
    p.add_argument("--max-draft-tokens", type=int, default=8)
    p.add_argument("--start-fraction", type=float, default=0.05)
    p.add_argument("--require-greedy", action=argparse.BooleanOptionalAction, default=True)
    args = p.parse_args(argv)
    logging.basicConfig(level=logging.INFO)
    proxy = Proxy(build_config(args))
    threading.Thread(target=uvicorn.run, args=(proxy.telemetry_app,),
                     kwargs={"host": args.host, "port": args.telemetry_port, "log_level": "info"},
                     daemon=True).start()
    uvicorn.run(proxy.app, host=args.host, port=args.port, log_level="info")


if __name__ == "__main__":
    main()
