"""Exclusive-GPU resource gate for latency-valid runs.

Parity with the reference's experiments/progressive_pd_resource_gate.py:
``nvidia-smi`` GPU and compute-process queries are parsed (the command runner
is injectable, so tests and dry runs never touch a GPU), and a requested GPU
fails the gate when it has any compute process, more memory in use than the
threshold, or utilisation above the threshold.  The gate only reads state;
it changes no GPU setting.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import subprocess
import sys
from dataclasses import asdict, dataclass
from typing import Any, Callable, Sequence

GPU_FIELDS = ("index", "uuid", "name", "memory.used", "memory.total", "utilization.gpu", "pstate",
              "temperature.gpu", "power.draw")


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
    compute_processes: tuple[dict[str, Any], ...]


def _rows(raw: str):
    return [r for r in csv.reader(io.StringIO(raw.strip())) if r]


def parse_gpu_query(raw: str) -> list[dict[str, Any]]:
    out = []
    for r in _rows(raw):
        if len(r) != len(GPU_FIELDS):
            raise ValueError(f"unexpected nvidia-smi GPU row: {r}")
        r = [x.strip() for x in r]
        out.append({"index": int(r[0]), "uuid": r[1], "name": r[2], "memory_used_mib": float(r[3]),
                    "memory_total_mib": float(r[4]), "utilization_pct": float(r[5]), "pstate": r[6],
                    "temperature_c": float(r[7]), "power_w": float(r[8])})
    if not out:
        raise ValueError("nvidia-smi returned no GPUs")
    return out


def parse_compute_query(raw: str) -> dict[str, list[dict[str, Any]]]:
    text = raw.strip()
    if not text or text.startswith("No running processes found"):
        return {}
    out: dict[str, list[dict[str, Any]]] = {}
    for r in _rows(text):
        if len(r) != 4:
            raise ValueError(f"unexpected nvidia-smi process row: {r}")
        uuid, pid, name, used = (x.strip() for x in r)
        out.setdefault(uuid, []).append({"pid": int(pid), "process_name": name,
                                         "used_gpu_memory_mib": None if used in ("N/A", "[N/A]") else float(used)})
    return out


def run_command(cmd: list[str]) -> str:
    return subprocess.run(cmd, check=True, capture_output=True, text=True).stdout


def inspect_gpus(*, command_runner: Callable[[list[str]], str] = run_command) -> list[GPUState]:
    gpus = parse_gpu_query(command_runner(["nvidia-smi", f"--query-gpu={','.join(GPU_FIELDS)}",
                                           "--format=csv,noheader,nounits"]))
    procs = parse_compute_query(command_runner(["nvidia-smi",
                                                "--query-compute-apps=gpu_uuid,pid,process_name,used_gpu_memory",
                                                "--format=csv,noheader,nounits"]))
    return [GPUState(**g, compute_processes=tuple(procs.get(g["uuid"], []))) for g in gpus]


def evaluate_exclusivity(states: Sequence[GPUState], requested: Sequence[int], *, max_used_memory_mib: float,
                         max_utilization_pct: float) -> dict[str, Any]:
    requested = tuple(requested)
    if not requested or len(requested) != len(set(requested)):
        raise ValueError("requested GPU indices must be a non-empty unique list")
    by = {s.index: s for s in states}
    missing = [i for i in requested if i not in by]
    if missing:
        raise ValueError(f"requested GPUs do not exist: {missing}")
    failures, selected = [], []
    for i in requested:
        s = by[i]
        selected.append(asdict(s))
        if s.compute_processes:
            failures.append({"gpu": i, "reason": "compute_processes_present", "processes": list(s.compute_processes)})
        if s.memory_used_mib > max_used_memory_mib:
            failures.append({"gpu": i, "reason": "memory_used_above_threshold", "observed_mib": s.memory_used_mib,
                             "threshold_mib": max_used_memory_mib})
        if s.utilization_pct > max_utilization_pct:
            failures.append({"gpu": i, "reason": "utilization_above_threshold", "observed_pct": s.utilization_pct,
                             "threshold_pct": max_utilization_pct})
    return {"status": "failed" if failures else "passed", "requested_gpus": list(requested),
            "thresholds": {"max_used_memory_mib": max_used_memory_mib, "max_utilization_pct": max_utilization_pct},
            "failures": failures, "gpus": selected}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="fail unless the requested GPUs are idle")
    p.add_argument("--gpus", required=True, help="comma-separated GPU indices")
    p.add_argument("--max-used-memory-mib", type=float, default=1024.0)
    p.add_argument("--max-utilization-pct", type=float, default=5.0)
    args = p.parse_args(argv)
    res = evaluate_exclusivity(inspect_gpus(), [int(x) for x in args.gpus.split(",")],
                               max_used_memory_mib=args.max_used_memory_mib,
                               max_utilization_pct=args.max_utilization_pct)
    print(json.dumps(res, indent=2))
    return 0 if res["status"] == "passed" else 2


if __name__ == "__main__":
    sys.exit(main())
