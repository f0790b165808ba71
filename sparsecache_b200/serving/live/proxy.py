"""1P1D proxy: one prefill per paired execution, store-completion gating, decode forwarding.

Behavioural parity with the reference's experiments/progressive_pd_proxy.py:
  * request validation of the proxy-owned ``sparsecache_*`` fields (mode
    baseline|progressive, visibility continuous|fixed_s1, max draft tokens,
    start fraction in (0, 1), request-scoped chunk priority, paired prefill
    group) and greedy-only requests (:137-214), written here as a table of
    field rules (``FIELD_RULES``) applied by ``ProxyRequest.parse``;
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
    """Identity of a prefill: sha256 of the canonical JSON of (endpoint, payload)."""
    canonical = json.dumps([endpoint, payload], sort_keys=True, separators=(",", ":"), ensure_ascii=False)
    return hashlib.sha256(canonical.encode("utf-8")).hexdigest()


def extract_seed_token(response: dict[str, Any]) -> int:
    """The producer's first generated token: ``choices[0].token_ids[0]`` of its response."""
    node: Any = response
    for key in ("choices", 0, "token_ids", 0):
        try:
            node = node[key]
        except (KeyError, IndexError, TypeError) as exc:
            raise RuntimeError("the prefill response has no choices[0].token_ids[0] "
                               "(the prefill worker must honour return_token_ids)") from exc
    if type(node) is not int:
        raise TypeError(f"the prefill seed token must be an integer, got {type(node).__name__}")
    return node


def _count(v: Any) -> bool:
    return type(v) is int and v >= 1


def _fraction(v: Any) -> bool:
    return type(v) in (int, float) and 0.0 < float(v) < 1.0


def _chunk_ids(v: Any) -> bool:
    return v is None or (type(v) is list and len(v) > 0 and all(type(c) is int and c >= 0 for c in v)
                         and len(set(v)) == len(v))


def _label(v: Any) -> bool:
    return v is None or (isinstance(v, str) and v.strip() != "")


@dataclass(frozen=True)
class FieldRule:
    """One proxy-owned request field: its default (from the config) and its check."""

    name: str
    default: Callable[[ProxyConfig], Any]
    valid: Callable[[Any], bool]
    expect: str


# the ``sparsecache_*`` fields a client may send; the proxy consumes them and
# never forwards them to a worker
FIELD_RULES = (
    FieldRule("sparsecache_mode", lambda c: c.default_mode, lambda v: v in ("baseline", "progressive"),
              "baseline or progressive"),
    FieldRule("sparsecache_visibility_mode", lambda c: c.default_visibility_mode,
              lambda v: v in ("continuous", "fixed_s1"), "continuous or fixed_s1"),
    FieldRule("sparsecache_max_draft_tokens", lambda c: c.max_draft_tokens, _count, "a positive integer"),
    FieldRule("sparsecache_start_fraction", lambda c: c.start_fraction, _fraction, "a number in (0, 1)"),
    FieldRule("sparsecache_priority_chunks", lambda c: None, _chunk_ids, "unique non-negative integers"),
    FieldRule("sparsecache_prefill_group", lambda c: None, _label, "a non-empty string"),
)


@dataclass(frozen=True)
class ProxyRequest:
    """A validated client request: the worker payload plus the proxy's settings."""

    payload: dict[str, Any]
    settings: dict[str, Any]

    @classmethod
    def parse(cls, request: dict[str, Any], config: ProxyConfig) -> "ProxyRequest":
        payload = dict(request)
        settings = {}
        for rule in FIELD_RULES:
            value = payload.pop(rule.name, rule.default(config))
            if not rule.valid(value):
                raise ValueError(f"{rule.name} must be {rule.expect}")
            settings[rule.name[len("sparsecache_"):]] = value
        if config.require_greedy and float(payload.get("temperature", 1.0)) != 0.0:
            raise ValueError("only greedy requests are served (the correctness gate needs temperature=0)")
        return cls(payload, settings)

    @property
    def mode(self) -> str:
        return self.settings["mode"]

    def prefill_payload(self) -> dict[str, Any]:
        """One non-streamed token whose id comes back (the seed)."""
        out = {k: v for k, v in self.payload.items() if k != "stream_options"}
        out.update(max_tokens=1, stream=False, return_token_ids=True)
        if "max_completion_tokens" in out:
            out["max_completion_tokens"] = 1
        return out

    def decode_payload(self, seed_token_id: int | None) -> dict[str, Any]:
        """The client request plus the proxy-owned ``kv_transfer_params`` entries."""
        out = dict(self.payload)
        client_params = dict(out.get("kv_transfer_params") or {})
        progressive = self.mode == "progressive"
        if progressive and seed_token_id is None:
            raise ValueError("progressive mode requires the exact prefiller seed")
        owned: dict[str, Any] = {"require_full_remote_kv": True}
        if progressive:
            owned["progressive_sparse_draft"] = {
                "seed_token_id": seed_token_id, "max_draft_tokens": self.settings["max_draft_tokens"],
                "start_fraction": float(self.settings["start_fraction"]),
                "visibility_mode": self.settings["visibility_mode"]}
        elif seed_token_id is not None:
            owned["producer_seed_token_id"] = seed_token_id
        taken = sorted(k for k in owned if k in client_params)
        if taken:
            raise ValueError(f"kv_transfer_params.{taken[0]} is proxy-owned")
        if progressive and self.settings["priority_chunks"] is not None:
            owned["progressive_priority_chunks"] = self.settings["priority_chunks"]
        if progressive or seed_token_id is not None:
            out["kv_transfer_params"] = {**client_params, **owned}
        return out


def prepare_requests(request: dict[str, Any], config: ProxyConfig, seed_token_id: int | None):
    """(prefill payload, decode payload, mode) of one client request."""
    parsed = ProxyRequest.parse(request, config)
    return parsed.prefill_payload(), parsed.decode_payload(seed_token_id), parsed.mode


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
