"""Exclusive-GPU gate (before a run) and exclusive-GPU monitor (during a run).

A latency cell is only valid when nothing else computes on its GPUs.  Two
checks enforce that, both read-only (no GPU setting is touched):

* ``evaluate_exclusivity`` (the gate) looks at one ``inspect_gpus`` snapshot
  and fails a requested GPU that has any compute process, more memory in use
  than a threshold, or utilisation above a threshold.
* ``ExclusivityMonitor`` (the runtime watch) polls during the run and reports
  the first compute process on a watched GPU that is not a descendant of the
  run's own service processes, or a watched GPU that disappeared; the launcher
  then stops the cell.

Behaviour parity: experiments/progressive_pd_resource_gate.py:16-183 (gate)
and experiments/run_progressive_pd_live_job.py:470-560 (runtime monitor) of
the reference.  The failure reasons and the verdict's ``status`` values are
the strings the reference's run records use.  ``nvidia-smi`` is reached only
through an injectable command runner, so tests and dry runs fake it.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import subprocess
import sys
import threading
import time
from dataclasses import asdict, dataclass, field
from typing import Any, Callable, Iterable, Sequence

Runner = Callable[[list[str]], str]


def _mib(text: str) -> float | None:
    return None if text in ("N/A", "[N/A]", "") else float(text)


# (nvidia-smi column, attribute, converter), in query order
GPU_COLUMNS = (
    ("index", "index", int),
    ("uuid", "uuid", str),
    ("name", "name", str),
    ("memory.used", "memory_used_mib", float),
    ("memory.total", "memory_total_mib", float),
    ("utilization.gpu", "utilization_pct", float),
    ("pstate", "pstate", str),
    ("temperature.gpu", "temperature_c", float),
    ("power.draw", "power_w", float),
)
APP_COLUMNS = (
    ("gpu_uuid", "gpu_uuid", str),
    ("pid", "pid", int),
    ("process_name", "process_name", str),
    ("used_gpu_memory", "used_gpu_memory_mib", _mib),
)


def run_command(cmd: list[str]) -> str:
    return subprocess.run(cmd, check=True, capture_output=True, text=True).stdout


def smi_table(text: str, columns: Sequence[tuple[str, str, Callable]], what: str) -> list[dict[str, Any]]:
    """Parse ``--format=csv,noheader,nounits`` output into dicts keyed by attribute name."""
    body = text.strip()
    if body.startswith("No running processes found"):
        return []
    records = []
    for fields in csv.reader(io.StringIO(body)):
        if not fields:
            continue
        if len(fields) != len(columns):
            raise ValueError(f"unexpected nvidia-smi {what} row: {fields}")
        records.append({attr: conv(raw.strip()) for (_, attr, conv), raw in zip(columns, fields)})
    return records


def _query(runner: Runner, target: str, columns) -> str:
    names = ",".join(c[0] for c in columns)
    return runner(["nvidia-smi", f"--query-{target}={names}", "--format=csv,noheader,nounits"])


def parse_gpu_query(raw: str) -> list[dict[str, Any]]:
    rows = smi_table(raw, GPU_COLUMNS, "GPU")
    if not rows:
        raise ValueError("nvidia-smi returned no GPUs")
    return rows


def parse_compute_query(raw: str) -> dict[str, list[dict[str, Any]]]:
    """Compute processes grouped by GPU uuid ({} when none run)."""
    by_gpu: dict[str, list[dict[str, Any]]] = {}
    for app in smi_table(raw, APP_COLUMNS, "process"):
        uuid = app.pop("gpu_uuid")
        by_gpu.setdefault(uuid, []).append(app)
    return by_gpu


@dataclass(frozen=True)
class GPUState:
    index: int
    uuid: str
    name: str
    memory_used_mib: float
    memory_total_mib: float
    utilization_pct: float
    pstate: str
    temperature_c: float
    power_w: float
    compute_processes: tuple[dict[str, Any], ...] = field(default=())


def inspect_gpus(*, command_runner: Runner = run_command) -> list[GPUState]:
    """One snapshot: every GPU with the compute processes running on it."""
    gpus = parse_gpu_query(_query(command_runner, "gpu", GPU_COLUMNS))
    apps = parse_compute_query(_query(command_runner, "compute-apps", APP_COLUMNS))
    return [GPUState(**g, compute_processes=tuple(apps.get(g["uuid"], ()))) for g in gpus]


@dataclass(frozen=True)
class Thresholds:
    max_used_memory_mib: float
    max_utilization_pct: float

    def violations(self, s: GPUState) -> list[dict[str, Any]]:
        out = []
        if s.compute_processes:
            out.append({"gpu": s.index, "reason": "compute_processes_present",
                        "processes": [dict(p) for p in s.compute_processes]})
        if s.memory_used_mib > self.max_used_memory_mib:
            out.append({"gpu": s.index, "reason": "memory_used_above_threshold",
                        "observed_mib": s.memory_used_mib, "threshold_mib": self.max_used_memory_mib})
        if s.utilization_pct > self.max_utilization_pct:
            out.append({"gpu": s.index, "reason": "utilization_above_threshold",
                        "observed_pct": s.utilization_pct, "threshold_pct": self.max_utilization_pct})
        return out


def _check_requested(requested: Sequence[int], known: Iterable[int]) -> tuple[int, ...]:
    req = tuple(int(i) for i in requested)
    if not req or len(set(req)) != len(req):
        raise ValueError("requested GPU indices must be a non-empty unique list")
    absent = sorted(set(req) - set(known))
    if absent:
        raise ValueError(f"requested GPUs do not exist: {absent}")
    return req


def evaluate_exclusivity(states: Sequence[GPUState], requested: Sequence[int], *, max_used_memory_mib: float,
                         max_utilization_pct: float) -> dict[str, Any]:
    """Gate verdict for the requested GPUs: ``status`` is "passed" or "failed"."""
    by_index = {s.index: s for s in states}
    req = _check_requested(requested, by_index)
    limits = Thresholds(max_used_memory_mib, max_utilization_pct)
    failures = [v for i in req for v in limits.violations(by_index[i])]
    return {
        "status": "failed" if failures else "passed",
        "checked_at_unix_ns": time.time_ns(),
        "requested_gpus": list(req),
        "thresholds": {**asdict(limits), "compute_processes_allowed": 0},
        "failures": failures,
        "gpus": [asdict(by_index[i]) for i in req],
    }


# --------------------------------------------------------------- runtime watch
def parent_pid(pid: int) -> int | None:
    """Parent of ``pid`` from /proc (None when the process is gone)."""
    try:
        with open(f"/proc/{pid}/stat") as f:
            stat = f.read()
    except OSError:
        return None
    # the command name (field 2) may hold spaces and parentheses: the fields
    # after its closing parenthesis are "state ppid ..."
    rest = stat[stat.rfind(")") + 2:].split()
    return int(rest[1]) if len(rest) > 1 else None


class ExclusivityMonitor:
    """Watch the run's GPUs for compute processes that the run did not start.

    ``service_roots`` are the pids of the processes this run launched (its
    workers and proxy); any compute process on a watched GPU whose ancestry
    does not reach one of them is foreign.  ``check()`` returns the first
    finding (or None); ``start(on_violation)`` polls in a daemon thread and
    calls ``on_violation(finding)`` once.
    """

    def __init__(self, gpus: Sequence[int], service_roots: Iterable[int], *,
                 command_runner: Runner = run_command, parent_of: Callable[[int], int | None] = parent_pid,
                 interval_s: float = 1.0) -> None:
        self.gpus = tuple(int(g) for g in gpus)
        self.roots = {int(p) for p in service_roots}
        self.runner = command_runner
        self.parent_of = parent_of
        self.interval_s = float(interval_s)
        self.samples = 0
        self.finding: dict[str, Any] | None = None
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    def add_root(self, pid: int) -> None:
        self.roots.add(int(pid))

    def owned(self, pid: int) -> bool:
        seen = set()
        while pid not in self.roots:
            if pid <= 1 or pid in seen:
                return False
            seen.add(pid)
            up = self.parent_of(pid)
            if up is None:
                return False
            pid = up
        return True

    def check(self) -> dict[str, Any] | None:
        states = {s.index: s for s in inspect_gpus(command_runner=self.runner)}
        self.samples += 1
        for g in self.gpus:
            s = states.get(g)
            if s is None:
                return {"gpu": g, "reason": "gpu_disappeared", "sample": self.samples}
            for proc in s.compute_processes:
                if not self.owned(int(proc["pid"])):
                    return {"gpu": g, "reason": "foreign_compute_process", "sample": self.samples, **proc}
        return None

    def start(self, on_violation: Callable[[dict[str, Any]], None]) -> None:
        def loop():
            while not self._stop.wait(self.interval_s):
                try:
                    found = self.check()
                except Exception as exc:  # noqa: BLE001 - an unreadable GPU state is itself a finding
                    found = {"reason": "monitor_query_failed", "error": f"{type(exc).__name__}: {exc}"}
                if found is not None:
                    self.finding = found
                    on_violation(found)
                    return

        self._thread = threading.Thread(target=loop, name="exclusive-gpu-monitor", daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=max(5.0, 2 * self.interval_s))


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="fail unless the requested GPUs are idle")
    p.add_argument("--gpus", required=True, help="comma-separated GPU indices")
    p.add_argument("--max-used-memory-mib", type=float, default=1024.0)
    p.add_argument("--max-utilization-pct", type=float, default=5.0)
    args = p.parse_args(argv)
    verdict = evaluate_exclusivity(inspect_gpus(), [int(x) for x in args.gpus.split(",")],
                                   max_used_memory_mib=args.max_used_memory_mib,
                                   max_utilization_pct=args.max_utilization_pct)
    print(json.dumps(verdict, indent=2))
    return 0 if verdict["status"] == "passed" else 2


if __name__ == "__main__":
    sys.exit(main())
