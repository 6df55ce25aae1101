"""Run the test suite and persist a receipt bound to the tested source tree (the counterpart of reference
scripts/verify.py).

``python -m reelcache_b200.verify --receipt receipt.json`` hashes every source of the package, its native
kernels and the tests (SHA-256 per file, one digest over the sorted map), runs ``pytest -m "not gpu"`` (or
``--gpu`` for the GPU tier) with a JUnit report, and writes a receipt with the tree digest, the per-test outcomes
and the environment. ``--check receipt.json`` recomputes the digest and fails when the tree changed since the
receipt was taken or the receipt records a failure.
"""

from __future__ import annotations

import argparse
import datetime
import hashlib
import json
import platform
import subprocess
import sys
import tempfile
import time
import xml.etree.ElementTree as ET
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PATTERNS = ("*.py", "*.cu", "*.cuh", "*.cpp", "*.h")


def source_identity(root: Path = ROOT) -> tuple[str, dict[str, str]]:
    files = set()
    for directory in ("reelcache_b200", "tests", "examples"):
        base = root / directory
        if base.exists():
            for pattern in PATTERNS:
                files.update(p for p in base.rglob(pattern) if "_build" not in p.parts and "__pycache__" not in p.parts)
    for name in ("bench.py", "__graft_entry__.py"):
        if (root / name).exists():
            files.add(root / name)
    identities = {str(p.relative_to(root)): hashlib.sha256(p.read_bytes()).hexdigest() for p in sorted(files)}
    digest = hashlib.sha256(json.dumps(identities, sort_keys=True, separators=(",", ":")).encode()).hexdigest()
    return digest, identities


def _outcomes(junit: Path) -> list[dict]:
    records = []
    for case in ET.parse(junit).getroot().iter("testcase"):
        status = "passed"
        detail = None
        for tag in ("failure", "error", "skipped"):
            node = case.find(tag)
            if node is not None:
                status = {"failure": "failed", "error": "error", "skipped": "skipped"}[tag]
                detail = (node.get("message") or "")[:500]
        records.append({"test": f"{case.get('classname')}::{case.get('name')}", "status": status,
                        "seconds": float(case.get("time") or 0.0), "detail": detail})
    return records


def run(receipt: Path, *, gpu: bool = False, extra: list[str] | None = None) -> int:
    digest, identities = source_identity()
    started = time.time()
    with tempfile.TemporaryDirectory() as scratch:
        junit = Path(scratch) / "junit.xml"
        command = [sys.executable, "-m", "pytest", str(ROOT / "tests"), "-q", "-m", "gpu" if gpu else "not gpu",
                   f"--junitxml={junit}", *(extra or [])]
        code = subprocess.call(command, cwd=ROOT)
        records = _outcomes(junit) if junit.exists() else []
    counts: dict[str, int] = {}
    for record in records:
        counts[record["status"]] = counts.get(record["status"], 0) + 1
    import torch
    body = {"schema": "reelcache_b200.verify_receipt.v1", "tree_sha256": digest, "files": len(identities),
            "tier": "gpu" if gpu else "cpu", "exit_code": code, "counts": counts, "tests": records,
            "started": datetime.datetime.fromtimestamp(started, datetime.timezone.utc).isoformat(),
            "seconds": time.time() - started,
            "environment": {"python": platform.python_version(), "torch": str(torch.__version__),
                            "cuda": str(torch.version.cuda), "machine": platform.machine()}}
    receipt.write_text(json.dumps(body, indent=1, sort_keys=True))
    print(json.dumps({"tree_sha256": digest, "exit_code": code, "counts": counts}))
    return code


def check(receipt: Path) -> int:
    body = json.loads(receipt.read_text())
    digest, _ = source_identity()
    if body.get("tree_sha256") != digest:
        print(f"stale receipt: tree {digest} differs from the tested {body.get('tree_sha256')}")
        return 2
    if body.get("exit_code") != 0 or body.get("counts", {}).get("failed") or body.get("counts", {}).get("error"):
        print("the receipt records failures")
        return 1
    print(f"receipt valid for tree {digest} ({body['counts']})")
    return 0


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--receipt", type=Path, default=ROOT / "verify_receipt.json")
    parser.add_argument("--gpu", action="store_true", help="run the GPU tier instead of the CPU tier")
    parser.add_argument("--check", type=Path, help="validate an existing receipt against the current tree")
    args, extra = parser.parse_known_args(argv)
    if args.check is not None:
        return check(args.check)
    return run(args.receipt, gpu=args.gpu, extra=extra)


if __name__ == "__main__":
    sys.exit(main())
