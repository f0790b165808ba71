"""Preregistered P/D experiment queue from an experiment matrix.

    python -m sparsecache_b200.pipelines.matrix_queue --matrix configs/pd_experiment_matrix.json \\
        --run-root runs/pd_matrix --output runs/pd_matrix/queue.json

Counterpart of the reference's experiments/build_iclr_pd_job_queue.py.  The
matrix JSON uses the reference's layout (``datasets[{name, path, available}]``,
``models[{name, path}]``, ``selection_split.progressive_focus_cells``
``{transport_gbps, draft_tokens, arrival_bundles}``, ``controlled_context``
``{paths, evidence_placement, requests_per_cell, primary_model_max_prompt_tokens}``,
``longbench_v2{path, available, llama31_8b_max_context_tokens}``).  Selection
is kept apart from confirmation:

  * ready jobs: a measurement-integrity gate (one isolated fixed first-stage
    cell, paired with the full target, checked by the latency-cell validator),
    the sparse-draft kernel crossover screen, and the continuous-visibility
    selection grid (models x link rates x draft horizons x arrival bundles on
    a 30-request split, each paired with the fixed first-stage control);
  * confirmation templates: quality per model x dataset, the controlled-context
    RULER cells and LongBench-v2, emitted with their policy fields unset and
    blocked until one policy is frozen from the selection results.

Every job names the commands of this package: a pack build
(``evaluation.cli``), the P/D run (``pipelines.pd --pack``) and, where
the reference has one, the validator.  The queue carries a sha256 over its jobs.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import re
from pathlib import Path
from typing import Any

PY = "python"
FREEZE_FIELDS = ("transport_gbps", "draft_tokens", "arrival_bundles", "priority_fraction", "page_tokens", "schedule")


def fractions_for_bundles(first_fraction: float, residual_bundles: int) -> str:
    """Cumulative stage fractions: the first tranche, then ``residual_bundles`` equal steps to 1."""
    if not 0.0 < first_fraction < 1.0 or residual_bundles < 1:
        raise ValueError("the first fraction must lie in (0, 1) and at least one residual bundle is needed")
    values = [first_fraction] + [first_fraction + (1.0 - first_fraction) * k / residual_bundles
                                 for k in range(1, residual_bundles + 1)]
    values[-1] = 1.0
    return ",".join(f"{v:.6f}" for v in values)


def slug(name: str) -> str:
    return re.sub(r"[^a-z0-9_]", "", name.lower().replace("-", "_").replace(".", ""))


def _pack_command(dataset: dict, model: dict, pack_dir: Path, *, requests: int | None, fmt: str = "longbench",
                  max_prompt_tokens: int = 32768, fixed_output_tokens: int | None = None) -> list[str]:
    cmd = [PY, "-m", "sparsecache_b200.evaluation.cli", "longbench-pack", "--dataset", str(dataset["path"]),
           "--dataset-name", dataset["name"], "--format", fmt, "--tokenizer", str(model["path"]),
           "--output-dir", str(pack_dir), "--max-prompt-tokens", str(max_prompt_tokens)]
    if requests is not None:
        cmd += ["--num-requests", str(requests)]
    if fixed_output_tokens is not None:
        cmd += ["--fixed-output-tokens", str(fixed_output_tokens)]
    return cmd


def _pd_command(pack_dir: Path, model: dict, output: Path, *, requests: int, fractions: str, drafts: int,
                bandwidth: float, paired_fixed_control: bool) -> list[str]:
    cmd = [PY, "-m", "sparsecache_b200.pipelines.pd", "--pack", str(pack_dir), "--model-dir", str(model["path"]),
           "--requests", str(requests), "--max-new-tokens", "64", "--context-page-tokens", "256",
           "--stage-fractions", fractions, "--draft-tokens", str(drafts), "--transport-gbps", str(bandwidth),
           "--schedule", "query", "--eager-serial-wire", "--require-exclusive-gpu", "--output", str(output)]
    if paired_fixed_control:
        cmd.append("--paired-fixed-control")
    return cmd


def build_matrix_queue(matrix: dict[str, Any], run_root: Path, *, matrix_path: str = "",
                       gate_dataset: str = "qmsum", selection_dataset: str = "qmsum") -> dict[str, Any]:
    run_root = Path(run_root)
    datasets = {d["name"]: d for d in matrix["datasets"]}
    for name in (gate_dataset, selection_dataset):
        if name not in datasets:
            raise ValueError(f"the matrix has no dataset {name!r}")
    if len(matrix["models"]) < 2:
        raise ValueError("the matrix needs a primary and a second model")
    primary, second = matrix["models"][:2]
    jobs: list[dict[str, Any]] = []

    gate_id = "gate_fixed_s1_" + slug(primary["name"]) + f"_{gate_dataset}_n100_bw100_s002_g6"
    gate_pack = run_root / "packs" / slug(primary["name"]) / f"{gate_dataset}_n100"
    gate_out = run_root / f"{gate_id}.jsonl"
    jobs.append({"id": gate_id, "phase": "measurement_integrity", "status": "ready",
                 "purpose": "one isolated fixed first-stage cell, paired with the full target",
                 "prepare": _pack_command(datasets[gate_dataset], primary, gate_pack, requests=100),
                 "command": _pd_command(gate_pack, primary, gate_out, requests=100, fractions="0.02,1.0", drafts=6,
                                        bandwidth=100, paired_fixed_control=False),
                 "validator": [PY, "-m", "sparsecache_b200.serving.live.validate", "latency-cell", str(gate_out),
                               "--expected", "100"]})
    kernel_id = "kernel_sparse_draft_crossover_8k"
    jobs.append({"id": kernel_id, "phase": "sparse_kernel_mechanism", "status": "ready",
                 "purpose": "per-token cost of a sparse-page draft step against the full-context step",
                 "command": [PY, "-m", "sparsecache_b200.pipelines.screens", "--contexts", "8192",
                             "--fractions", "0.02,0.25,0.5,0.75", "--draft-tokens", "8"],
                 "stdout": str(run_root / f"{kernel_id}.json")})
    focus = matrix["selection_split"]["progressive_focus_cells"]
    for model in (primary, second):
        pack = run_root / "packs" / slug(model["name"]) / f"{selection_dataset}_n30"
        for bw in focus["transport_gbps"]:
            for drafts in focus["draft_tokens"]:
                for bundles in focus["arrival_bundles"]:
                    jid = f"select_{slug(model['name'])}_{selection_dataset}_n30_bw{bw}_g{drafts}_b{bundles}"
                    jobs.append({"id": jid, "phase": "continuous_policy_selection", "status": "ready",
                                 "purpose": "continuous page visibility against the fixed first stage",
                                 "prepare": _pack_command(datasets[selection_dataset], model, pack, requests=30),
                                 "command": _pd_command(pack, model, run_root / f"{jid}.jsonl", requests=30,
                                                        fractions=fractions_for_bundles(0.02, bundles),
                                                        drafts=drafts, bandwidth=bw, paired_fixed_control=True),
                                 "model": model["name"], "bandwidth_gbps": bw, "draft_tokens": drafts,
                                 "residual_bundles": bundles})
    templates: list[dict[str, Any]] = []
    for model in (primary, second):
        for d in matrix["datasets"]:
            templates.append({"id": f"quality_{model['name']}_{d['name']}", "dataset": d["path"],
                              "dataset_format": "longbench", "model": model["path"],
                              "sample_count": d.get("available"), "official_output_length": True,
                              "max_context_tokens": 32768})
    cc = matrix.get("controlled_context", {})
    for nominal, path in cc.get("paths", {}).items():
        for placement in cc.get("evidence_placement", ()):
            templates.append({"id": f"ruler_{slug(primary['name'])}_{nominal}_{placement}", "dataset": path,
                              "dataset_format": "ruler", "model": primary["path"],
                              "sample_count": cc.get("requests_per_cell"),
                              "ruler_placement": (f"evidence_{placement}" if placement in ("first", "uniform", "last")
                                                  else placement),
                              "official_output_length": True,
                              "max_prompt_tokens": cc.get("primary_model_max_prompt_tokens")})
    if "longbench_v2" in matrix:
        lb2 = matrix["longbench_v2"]
        templates.append({"id": f"longbench_v2_{slug(primary['name'])}_all", "dataset": lb2["path"],
                          "dataset_format": "longbench_v2", "model": primary["path"],
                          "sample_count": lb2.get("available"), "official_output_length": True,
                          "max_context_tokens": lb2.get("llama31_8b_max_context_tokens")})
    ids = [j["id"] for j in jobs]
    if len(ids) != len(set(ids)):
        raise ValueError("duplicate job ids")
    return {"schema_version": 1, "matrix": matrix_path, "selection_is_preregistered": True, "ready_jobs": jobs,
            "jobs_sha256": hashlib.sha256(json.dumps(jobs, sort_keys=True).encode()).hexdigest(),
            "confirmation_policy": {"status": "blocked_on_continuous_policy_selection",
                                    "freeze_fields": list(FREEZE_FIELDS), "templates": templates},
            "counts": {"ready": len(jobs),
                       **{ph: sum(j["phase"] == ph for j in jobs) for ph in
                          ("measurement_integrity", "continuous_policy_selection", "sparse_kernel_mechanism")},
                       "confirmation_templates": len(templates)}}


def main(argv=None) -> dict[str, Any]:
    p = argparse.ArgumentParser()
    p.add_argument("--matrix", type=Path, required=True)
    p.add_argument("--run-root", type=Path, required=True)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--gate-dataset", default="qmsum")
    p.add_argument("--selection-dataset", default="qmsum")
    a = p.parse_args(argv)
    queue = build_matrix_queue(json.loads(a.matrix.read_text(encoding="utf-8")), a.run_root,
                               matrix_path=str(a.matrix.resolve()), gate_dataset=a.gate_dataset,
                               selection_dataset=a.selection_dataset)
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(queue, indent=2, ensure_ascii=False) + "\n", encoding="utf-8")
    print(json.dumps(queue["counts"]))
    return queue


if __name__ == "__main__":
    main()
