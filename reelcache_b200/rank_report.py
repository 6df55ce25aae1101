"""Rank study report of an archived lineage (the counterpart of the reference's rank-study / report / compare
scripts, scripts/ in the reference tree): for every node on a head's path, the per-matrix ranks the rank method
chose, the energy each record reached against its target, the post-codec error, the bytes the node added and
the compression ratio against the native bf16 matrices; ``compare`` puts two reports side by side (for example
two energy targets or two solvers on the same history).

    python -m reelcache_b200.rank_report --store DIR --branch main [--json]
    python -m reelcache_b200.rank_report --store DIR --node <ref> --compare-store DIR2 --compare-node <ref>
"""

from __future__ import annotations

import argparse
import json
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from .store import ObjectStore
from .types import ModelIdentity, entry_parts


@dataclass
class NodeReport:
    node_ref: str
    chunk_id: str
    tokens: int
    records: int
    ranks: dict = field(default_factory=dict)           # target -> [rank per layer]
    energy: dict = field(default_factory=dict)          # target -> {"min_stored": .., "targets_met": ..}
    post_codec_error: dict = field(default_factory=dict)
    bytes: dict = field(default_factory=dict)
    native_bytes: int = 0

    @property
    def ratio(self) -> float | None:
        total = self.bytes.get("total_bytes", 0)
        return self.native_bytes / total if total else None

    def to_dict(self) -> dict:
        return {"node": self.node_ref, "chunk": self.chunk_id, "tokens": self.tokens, "records": self.records,
                "ranks": self.ranks, "energy": self.energy, "post_codec_error": self.post_codec_error,
                "bytes": self.bytes, "native_bytes": self.native_bytes,
                "compression_ratio": None if self.ratio is None else round(self.ratio, 2)}


def _runtime(store: ObjectStore, head_ref: str | None = None, branch: str | None = None):
    """A read-only lineage view of ``store`` for the model that wrote ``head_ref`` (or ``branch``'s head);
    returns ``(runtime, head_ref)``."""
    from .lineage import LineageRuntime
    if head_ref is None:
        placeholder = ModelIdentity("report", "report", 1, 1, "BTHD", "bfloat16")
        head_ref = LineageRuntime(store, placeholder).lineage_head(branch)
    identity = ModelIdentity.from_dict(store.get_manifest(head_ref)["model"])
    return LineageRuntime(store, identity), head_ref


def node_report(runtime, node_ref: str) -> NodeReport:
    node = runtime.load_node(node_ref)
    report = NodeReport(node_ref, node.chunk_id, node.token_end - node.token_start, len(node.matrix_records))
    stored: dict[str, list] = {}
    met: dict[str, list] = {}
    errors: dict[str, list] = {}
    layers: dict[str, dict[int, int]] = {}
    native = 0
    for entry, record_ref in node.matrix_records:
        key, _ = entry_parts(entry)
        record = runtime.load_record(record_ref)
        ctx = record.context
        native += ctx.token_count * ctx.model.channels_for(key.target) * 2
        if record.rank_view is not None:
            layers.setdefault(key.target, {})[key.layer] = int(record.rank_view)
        if record.energy is not None:
            stored.setdefault(key.target, []).append(record.energy.stored_factor_energy)
            met.setdefault(key.target, []).append(record.energy.stored_factor_energy >= record.energy.target)
            if record.energy.post_codec_relative_error is not None:
                errors.setdefault(key.target, []).append(record.energy.post_codec_relative_error)
    for target, by_layer in layers.items():
        report.ranks[target] = [by_layer[layer] for layer in sorted(by_layer)]
    for target, values in stored.items():
        report.energy[target] = {"min_stored": round(float(min(values)), 6), "mean_stored": round(float(np.mean(values)), 6),
                                 "targets_met": int(sum(met[target])), "records": len(values)}
    for target, values in errors.items():
        report.post_codec_error[target] = {"max": float(max(values)), "mean": float(np.mean(values))}
    report.bytes = runtime.node_storage(node_ref)
    report.native_bytes = native
    return report


def lineage_report(runtime, head_ref: str) -> dict[str, Any]:
    """Reports of every node on ``head_ref``'s path that holds matrices (root first) and their totals."""
    nodes = [node_report(runtime, ref) for ref, node, _ in runtime.node_path(head_ref) if node.matrix_records]
    ranks = {t: [r for n in nodes for r in n.ranks.get(t, [])] for t in ("K", "V")}
    total_bytes = sum(n.bytes.get("total_bytes", 0) for n in nodes)
    native = sum(n.native_bytes for n in nodes)
    summary = {"nodes": len(nodes), "total_bytes": total_bytes, "native_bytes": native,
               "compression_ratio": round(native / total_bytes, 2) if total_bytes else None}
    for target, values in ranks.items():
        if values:
            summary[f"rank_{target}"] = {"min": int(min(values)), "mean": round(float(np.mean(values)), 2),
                                         "max": int(max(values))}
    return {"head": head_ref, "summary": summary, "nodes": [n.to_dict() for n in nodes]}


def compare(a: dict, b: dict) -> dict:
    """Side-by-side totals of two lineage reports and the per-node rank and byte deltas (b - a)."""
    rows = []
    for na, nb in zip(a["nodes"], b["nodes"]):
        row = {"chunk": na["chunk"], "bytes_a": na["bytes"].get("total_bytes"), "bytes_b": nb["bytes"].get("total_bytes")}
        for target in ("K", "V"):
            ra, rb = na["ranks"].get(target), nb["ranks"].get(target)
            if ra and rb:
                row[f"mean_rank_{target}_a"] = round(float(np.mean(ra)), 2)
                row[f"mean_rank_{target}_b"] = round(float(np.mean(rb)), 2)
        rows.append(row)
    return {"a": a["summary"], "b": b["summary"], "nodes": rows}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--store", required=True)
    ap.add_argument("--branch")
    ap.add_argument("--node")
    ap.add_argument("--compare-store")
    ap.add_argument("--compare-branch")
    ap.add_argument("--compare-node")
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args(argv)

    def load(store_path, branch, node):
        store = ObjectStore(store_path)
        runtime, head = _runtime(store, node, branch)
        return store, lineage_report(runtime, head)

    store, report = load(args.store, args.branch, args.node)
    try:
        if args.compare_store or args.compare_node or args.compare_branch:
            other_store, other = load(args.compare_store or args.store, args.compare_branch or args.branch,
                                      args.compare_node)
            try:
                report = compare(report, other)
            finally:
                other_store.close()
        if args.json or "a" in report:
            print(json.dumps(report, indent=1))
        else:
            summary = report["summary"]
            print(f"head {report['head']}: {summary['nodes']} nodes, {summary['total_bytes']} bytes stored for "
                  f"{summary['native_bytes']} native bytes (x{summary['compression_ratio']})")
            for node in report["nodes"]:
                ranks = {t: round(float(np.mean(v)), 1) for t, v in node["ranks"].items()}
                print(f"  {node['chunk']:>12}  tokens {node['tokens']:>6}  mean rank {ranks}  "
                      f"bytes {node['bytes'].get('total_bytes')}  x{node['compression_ratio']}")
    finally:
        store.close()


if __name__ == "__main__":
    main()
