"""Runs one candidate kernel through the worker in a child process with a time limit
(kernelpilot/agent/sandbox.py:24-64: same call and results).

This is isolation, not a security boundary: the child can reach the file system. It
keeps a hang, a segfault or a GPU fault in generated code away from the caller, and
gives every candidate a fresh CUDA context. The child runs in a session of its own,
so a time-out ends the whole process group (the worker and any compiler processes it
started), not only the worker.
"""

from __future__ import annotations

import json
import os
import signal
import subprocess
import sys
import tempfile
import time
from pathlib import Path

from .result import EvalResult

REPO_ROOT = Path(__file__).resolve().parents[2]


def _tail(s: str, n: int = 4000) -> str:
    return s if len(s) <= n else "...(truncated)...\n" + s[-n:]


def _text(b) -> str:
    if b is None:
        return ""
    return b.decode(errors="replace") if isinstance(b, bytes) else b


def run_candidate(code: str, kernel: str, lang: str = "cuda", dtype: str = "float32",
                  timeout_s: float = 300.0, bench_shapes: list[tuple] | None = None,
                  workdir: Path | None = None) -> EvalResult:
    tmp = Path(workdir or tempfile.mkdtemp(prefix="kpb_cand_"))
    tmp.mkdir(parents=True, exist_ok=True)
    code_path = tmp / "candidate.cu"
    code_path.write_text(code)
    out_path = tmp / "result.json"
    if out_path.exists():
        out_path.unlink()
    cmd = [sys.executable, "-m", "kernelpilot_b200.agent.worker", "--kernel", kernel,
           "--lang", lang, "--dtype", dtype, "--code", str(code_path), "--out", str(out_path),
           "--build-dir", str(tmp / "build")]
    if bench_shapes:
        cmd += ["--bench-shapes", json.dumps([list(s) for s in bench_shapes])]
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join(filter(None, [str(REPO_ROOT), env.get("PYTHONPATH")]))
    env.setdefault("TORCH_EXTENSIONS_DIR", str(tmp / "torch_ext"))
    t0 = time.monotonic()
    proc = subprocess.Popen(cmd, cwd=tmp, env=env, stdout=subprocess.PIPE,
                            stderr=subprocess.STDOUT, start_new_session=True)
    try:
        out, _ = proc.communicate(timeout=timeout_s)
    except subprocess.TimeoutExpired:
        try:
            os.killpg(proc.pid, signal.SIGKILL)
        except ProcessLookupError:
            pass
        out, _ = proc.communicate()
        return EvalResult(stage="timeout",
                          error=f"candidate did not finish within {timeout_s:g} s "
                                "(a hang, a deadlock, or far too slow)",
                          compile_log=_tail(_text(out)), duration_s=time.monotonic() - t0)
    output = _tail(_text(out))
    if not out_path.exists():
        return EvalResult(stage="crash",
                          error=f"worker exited with code {proc.returncode} and no result "
                                f"(segfault or GPU fault?)\n{output}",
                          duration_s=time.monotonic() - t0)
    res = EvalResult.from_dict(json.loads(out_path.read_text()))
    if not res.compile_log:
        res.compile_log = output
    res.duration_s = time.monotonic() - t0
    return res
