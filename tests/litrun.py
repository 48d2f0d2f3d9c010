"""A small lit-style runner: executes the `// RUN:` lines of an MLIR test file
with `tensixflow-opt` bound to this backend's `tfb200-opt` and `FileCheck` bound
to the FileCheck binary shipped in the triton wheel. `split-file %s %t` is done
in Python. RUN lines that use flags this backend does not implement are
reported as skipped.
"""

from __future__ import annotations

import os
import re
import subprocess
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
TOOL = ROOT / "tt-flow_b200" / "bin" / "tfb200-opt"
SUPPORTED = {"--tensixflow-device=b200", "--tensixflow-fuse-rmsnorm-matmul", "--tensixflow-plan-noc-sharding",
             "--tensixflow-allocate-circular-buffers", "--tensixflow-to-json", "-verify-diagnostics",
             "--tensixflow-import-ttir", "--allow-unregistered-dialect", "--canonicalize",
             "--tensixflow-canonicalize"}


def filecheck() -> str | None:
    try:
        import triton

        p = Path(triton.__file__).parent / "FileCheck"
        return str(p) if p.exists() else None
    except Exception:
        return None


def split_file(text: str, out: Path) -> None:
    parts = re.split(r"^//--- (\S+)\n", text, flags=re.M)
    out.mkdir(parents=True, exist_ok=True)
    for i in range(1, len(parts), 2):
        # keep line numbers of each part relative to its own file (as split-file does)
        (out / parts[i]).write_text(parts[i + 1])


def run_file(path: Path) -> dict:
    text = path.read_text()
    runs = [m.group(1).strip() for m in re.finditer(r"^// RUN:(.*)$", text, flags=re.M)]
    fc = filecheck()
    res = {"ran": 0, "skipped": [], "failed": []}
    with tempfile.TemporaryDirectory() as td:
        t = Path(td) / "t"
        for r in runs:
            if r.startswith("split-file"):
                split_file(text, t)
                continue
            head = re.sub(r"^not\s+", "", r.split("|")[0].strip())
            if not head.startswith("tensixflow-opt") or fc is None:
                # only invocations of the compiler are run (not checks on emitted
                # TT-Metalium project files)
                res["skipped"].append(r)
                continue
            tool_flags = {f for f in head.split()[1:] if f.startswith("-") and f not in ("-o",)
                          and not f.startswith("--tensixflow-device=")}
            if not tool_flags <= SUPPORTED:
                res["skipped"].append(r)
                continue
            cmd = r.replace("%s", str(path)).replace("%t", str(t)).replace("%S", str(path.parent))
            cmd = re.sub(r"\btensixflow-opt\b", str(TOOL), cmd)
            cmd = re.sub(r"\bFileCheck\b", fc, cmd)
            if re.match(r"^not\s+", cmd):
                # lit's `not` inverts the status of its own command only, not the pipeline's
                first, sep, rest = cmd.partition("|")
                cmd = "( ! " + re.sub(r"^not\s+", "", first).strip() + " )" + (" |" + rest if sep else "")
            p = subprocess.run(["bash", "-o", "pipefail", "-c", cmd], capture_output=True, text=True,
                               env=dict(os.environ))
            res["ran"] += 1
            if p.returncode != 0:
                res["failed"].append((r, p.stdout[-2000:] + p.stderr[-2000:]))
    return res
