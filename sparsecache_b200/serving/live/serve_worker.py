"""Run one worker role of the live harness as an HTTP server.

    python -m sparsecache_b200.serving.live.serve_worker --role prefill --port 8100 \
        --telemetry-url http://127.0.0.1:5768/api/v1/telemetry [--toy | --model llama3-8b]

``--toy`` serves the deterministic CPU worker (harness checks without a
GPU); otherwise the engine of ``--model`` (random-init weights, seeded)
serves on the visible GPU.
"""
from __future__ import annotations

import argparse
from pathlib import Path


def main(argv=None) -> None:
    import uvicorn

    from .worker import EngineWorker, TelemetrySink, ToyWorker, make_app

    p = argparse.ArgumentParser()
    p.add_argument("--role", choices=("prefill", "decode"), required=True)
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, required=True)
    p.add_argument("--telemetry-url")
    p.add_argument("--telemetry-dir", type=Path)
    p.add_argument("--toy", action="store_true")
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--capacity", type=int, default=32768)
    a = p.parse_args(argv)
    sink = TelemetrySink(a.telemetry_dir)
    if a.toy:
        worker = ToyWorker(telemetry=sink)
    else:
        from ...config import get_model_config
        from ...models.engine import B200Engine

        engine = B200Engine.random(get_model_config(a.model), seed=0, device="cuda",
                                   max_positions=a.capacity + 64)
        worker = EngineWorker(engine, capacity=a.capacity, telemetry=sink)
    uvicorn.run(make_app(worker, a.role, telemetry_url=a.telemetry_url), host=a.host, port=a.port,
                log_level="info")


if __name__ == "__main__":
    main()
