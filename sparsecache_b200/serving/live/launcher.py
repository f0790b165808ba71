"""Fail-closed launcher of one preregistered live job.

Parity with the reference's experiments/run_progressive_pd_live_job.py
(:84-777): the job is loaded from a hash-checked queue and its pack hashes
are re-verified; the exclusive-GPU gate must pass for every GPU the job
uses; every port must be free; the prefill worker, decode worker and proxy
start in their own process groups with logs in the run directory; the
launcher waits for their health endpoints (and stops at the first fatal
startup log line); then it runs the paired benchmark client, aggregates,
verifies the input trace and writes a run manifest.  While the services run,
an optional exclusive-GPU monitor polls the GPUs and stops the cell at the
first compute process that is not one of the launched services' own.  Any failure stops all
the launched process groups (by the group ids this launcher created) and
leaves a manifest with the failure reason.
"""
from __future__ import annotations

import json
import os
import signal
import socket
import subprocess
import sys
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Sequence

FATAL_MARKERS = ("Traceback (most recent call last)", "CUDA error", "out of memory", "Address already in use")


@dataclass
class ManagedProcess:
    name: str
    popen: subprocess.Popen
    log: Path


def assert_ports_free(host: str, ports: Sequence[int]) -> None:
    busy = []
    for p in ports:
        with socket.socket() as s:
            s.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            try:
                s.bind((host, p))
            except OSError:
                busy.append(p)
    if busy:
        raise RuntimeError(f"ports already in use: {busy}")


def spawn(name: str, argv: Sequence[str], log_dir: Path, env: dict | None = None) -> ManagedProcess:
    log_dir.mkdir(parents=True, exist_ok=True)
    log = log_dir / f"{name}.log"
    f = open(log, "w")
    p = subprocess.Popen(list(argv), stdout=f, stderr=subprocess.STDOUT, env={**os.environ, **(env or {})},
                         start_new_session=True)  # own process group, stopped as a unit
    return ManagedProcess(name, p, log)


def tail(path: Path, chars: int = 4000) -> str:
    try:
        return path.read_text(errors="replace")[-chars:]
    except FileNotFoundError:
        return ""


def fatal_startup(procs: Sequence[ManagedProcess]) -> None:
    for mp in procs:
        if mp.popen.poll() is not None:
            raise RuntimeError(f"{mp.name} exited with {mp.popen.returncode} during startup:\n{tail(mp.log)}")
        text = tail(mp.log, 20000)
        for marker in FATAL_MARKERS:
            if marker in text:
                raise RuntimeError(f"{mp.name} logged a fatal startup error ({marker}):\n{tail(mp.log)}")


def wait_http(url: str, procs: Sequence[ManagedProcess], timeout_s: float, get: Callable[[str], int] | None = None):
    import httpx

    get = get or (lambda u: httpx.get(u, timeout=2.0, trust_env=False).status_code)
    deadline = time.monotonic() + timeout_s
    while time.monotonic() < deadline:
        fatal_startup(procs)
        try:
            if get(url) == 200:
                return
        except Exception:  # noqa: BLE001  (not up yet)
            pass
        time.sleep(0.5)
    raise TimeoutError(f"{url} not healthy after {timeout_s}s")


def stop(procs: Sequence[ManagedProcess], timeout_s: float = 30.0) -> None:
    """SIGTERM then SIGKILL each launched process group (only the groups created here)."""
    for mp in procs:
        if mp.popen.poll() is None:
            try:
                os.killpg(mp.popen.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
    deadline = time.monotonic() + timeout_s
    for mp in procs:
        left = max(0.0, deadline - time.monotonic())
        try:
            mp.popen.wait(timeout=left)
        except subprocess.TimeoutExpired:
            try:
                os.killpg(mp.popen.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            mp.popen.wait()


def launch_spec(job: dict, *, host: str = "127.0.0.1", ports: dict | None = None, gpus: Sequence[int] = (0, 1),
                worker_module: str = "sparsecache_b200.serving.live.serve_worker") -> list[dict]:
    ports = ports or {"proxy": 8000, "telemetry": 5768, "prefill": 8100, "decode": 8200}
    py = sys.executable
    tele = f"http://{host}:{ports['telemetry']}/api/v1/telemetry"
    return [
        {"name": "prefill", "argv": [py, "-m", worker_module, "--role", "prefill", "--host", host, "--port",
                                     str(ports["prefill"]), "--telemetry-url", tele],
         "env": {"CUDA_VISIBLE_DEVICES": str(gpus[0])}, "health": f"http://{host}:{ports['prefill']}/health"},
        {"name": "decode", "argv": [py, "-m", worker_module, "--role", "decode", "--host", host, "--port",
                                    str(ports["decode"])],
         "env": {"CUDA_VISIBLE_DEVICES": str(gpus[-1])}, "health": f"http://{host}:{ports['decode']}/health"},
        {"name": "proxy", "argv": [py, "-m", "sparsecache_b200.serving.live.proxy", "--host", host, "--port",
                                   str(ports["proxy"]), "--telemetry-port", str(ports["telemetry"]),
                                   "--prefiller-url", f"http://{host}:{ports['prefill']}",
                                   "--decoder-url", f"http://{host}:{ports['decode']}",
                                   "--max-draft-tokens", str(job.get("max_draft_tokens", 8))],
         "env": {}, "health": f"http://{host}:{ports['proxy']}/health"},
    ]


def execute(job: dict, run_dir: Path, *, gate: Callable[[], dict] | None = None, host: str = "127.0.0.1",
            ports: dict | None = None, startup_timeout_s: float = 600.0,
            run_client: Callable[[], Any] | None = None,
            monitor: Callable[[Sequence[int]], Any] | None = None,
            spec: list[dict] | None = None) -> dict[str, Any]:
    """Run one job fail-closed; returns (and writes) the run manifest.

    ``monitor(service_pids)`` builds the runtime exclusive-GPU watch (a
    ``gate.ExclusivityMonitor``) once the services run; the first foreign
    compute process it sees stops every launched process group and fails
    the run (reference run_progressive_pd_live_job.py:524-560).
    """
    from .queue import validate_pack_hashes

    run_dir.mkdir(parents=True, exist_ok=True)
    manifest: dict[str, Any] = {"job_id": job["job_id"], "started_at": time.time(), "status": "failed"}
    procs: list[ManagedProcess] = []
    watch = None
    try:
        manifest["pack_hashes"] = validate_pack_hashes(job)
        if gate is not None:
            res = gate()
            manifest["resource_gate"] = res
            if res.get("status") != "passed":
                raise RuntimeError("exclusive-GPU gate failed")
        spec = spec if spec is not None else launch_spec(job, host=host, ports=ports)
        health = [s["health"] for s in spec if s.get("health")]
        assert_ports_free(host, [int(a.rsplit(":", 1)[1].split("/")[0]) for a in health])
        for s in spec:
            procs.append(spawn(s["name"], s["argv"], run_dir / "logs", s["env"]))
        if monitor is not None:
            watch = monitor([mp.popen.pid for mp in procs])
            watch.start(lambda finding: stop(procs, timeout_s=10.0))
        for s in spec:
            if s.get("health"):
                wait_http(s["health"], procs, startup_timeout_s)
        if run_client is not None:
            manifest["client"] = run_client()
        if watch is not None and watch.finding is not None:
            raise RuntimeError("interference")
        manifest["status"] = "completed"
    except Exception as exc:  # noqa: BLE001
        manifest["error"] = f"{type(exc).__name__}: {exc}"
    finally:
        if watch is not None:
            watch.stop()
            manifest["runtime_monitor"] = {"samples": watch.samples, "finding": watch.finding}
            if watch.finding is not None:
                manifest["status"] = "failed"
                manifest["error"] = ("runtime exclusive-GPU monitor detected interference: "
                                     + json.dumps(watch.finding, default=str))
        stop(procs)
        manifest["finished_at"] = time.time()
        (run_dir / "run_manifest.json").write_text(json.dumps(manifest, indent=2, default=str) + "\n")
    return manifest
