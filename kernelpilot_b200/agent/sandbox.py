"""Runs one candidate kernel through the worker in a child process with a deadline.

Same call and results as kernelpilot/agent/sandbox.py:24-64 (``run_candidate`` ->
``EvalResult``; the stages "timeout" and "crash" for a child that overran or died).
The mechanism is this module's own:

* the child runs in a session of its own, so the deadline ends the whole process
  group (the worker and the nvcc/ninja processes it started), not only the worker;
* the result travels back over a pipe handed to the child (``--result-fd``), not a
  file that a previous run could have left behind;
* the child's merged stdout/stderr is drained while it runs, through a selector with
  the deadline as its timeout, and only the last ``LOG_TAIL`` bytes are kept, so a
  candidate that prints without end neither blocks on a full pipe nor fills memory.

This is isolation, not a security boundary: the child can reach the file system. It
keeps a hang, a segfault or a GPU fault in generated code away from the caller, and
gives every candidate a fresh CUDA context.
"""

from __future__ import annotations

import json
import os
import selectors
import signal
import subprocess
import sys
import tempfile
import time
from pathlib import Path

from .result import EvalResult

REPO_ROOT = Path(__file__).resolve().parents[2]
LOG_TAIL = 4000


class _Tail:
    """The last ``limit`` bytes written to it."""

    def __init__(self, limit: int):
        self.limit, self.buf, self.dropped = limit, bytearray(), False

    def add(self, data: bytes) -> None:
        self.buf += data
        if len(self.buf) > 2 * self.limit:
            del self.buf[:-self.limit]
            self.dropped = True

    def text(self) -> str:
        data = bytes(self.buf[-self.limit:])
        head = "...(truncated)...\n" if self.dropped or len(self.buf) > self.limit else ""
        return head + data.decode(errors="replace")


def _worker_cmd(code_path: Path, kernel: str, lang: str, dtype: str, result_fd: int,
                build_dir: Path, bench_shapes) -> list[str]:
    cmd = [sys.executable, "-m", "kernelpilot_b200.agent.worker", "--kernel", kernel,
           "--lang", lang, "--dtype", dtype, "--code", str(code_path),
           "--result-fd", str(result_fd), "--build-dir", str(build_dir)]
    if bench_shapes:
        cmd += ["--bench-shapes", json.dumps([list(s) for s in bench_shapes])]
    return cmd


def _drain(proc: subprocess.Popen, result_r: int, deadline: float
           ) -> tuple[bool, _Tail, bytes]:
    """Read the child's output and result pipe until both close or the deadline
    passes. Returns (finished in time, output tail, result bytes)."""
    log, result = _Tail(LOG_TAIL), bytearray()
    sel = selectors.DefaultSelector()
    sel.register(proc.stdout, selectors.EVENT_READ, "log")
    sel.register(result_r, selectors.EVENT_READ, "result")
    open_streams = 2
    while open_streams:
        left = deadline - time.monotonic()
        if left <= 0:
            sel.close()
            return False, log, bytes(result)
        for key, _ in sel.select(timeout=min(left, 1.0)):
            chunk = os.read(key.fd, 65536)
            if not chunk:
                sel.unregister(key.fileobj)
                open_streams -= 1
            elif key.data == "log":
                log.add(chunk)
            else:
                result += chunk
    sel.close()
    left = max(0.0, deadline - time.monotonic())
    try:
        proc.wait(timeout=left)
    except subprocess.TimeoutExpired:
        return False, log, bytes(result)
    return True, log, bytes(result)


def run_candidate(code: str, kernel: str, lang: str = "cuda", dtype: str = "float32",
                  timeout_s: float = 300.0, bench_shapes: list[tuple] | None = None,
                  workdir: Path | None = None) -> EvalResult:
    tmp = Path(workdir or tempfile.mkdtemp(prefix="kpb_cand_"))
    tmp.mkdir(parents=True, exist_ok=True)
    code_path = tmp / "candidate.cu"
    code_path.write_text(code)
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join(filter(None, [str(REPO_ROOT), env.get("PYTHONPATH")]))
    env.setdefault("TORCH_EXTENSIONS_DIR", str(tmp / "torch_ext"))
    result_r, result_w = os.pipe()
    t0 = time.monotonic()
    try:
        proc = subprocess.Popen(
            _worker_cmd(code_path, kernel, lang, dtype, result_w, tmp / "build", bench_shapes),
            cwd=tmp, env=env, stdin=subprocess.DEVNULL, stdout=subprocess.PIPE,
            stderr=subprocess.STDOUT, pass_fds=(result_w,), start_new_session=True)
    finally:
        os.close(result_w)  # the child holds its own copy; EOF comes when it exits
    try:
        in_time, log, raw = _drain(proc, result_r, t0 + timeout_s)
        if not in_time:
            try:
                os.killpg(proc.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            proc.wait()
            return EvalResult(stage="timeout",
                              error=f"candidate did not finish within {timeout_s:g} s "
                                    "(a hang, a deadlock, or far too slow)",
                              compile_log=log.text(), duration_s=time.monotonic() - t0)
    finally:
        os.close(result_r)
        if proc.stdout:
            proc.stdout.close()
    elapsed = time.monotonic() - t0
    try:
        res = EvalResult.from_dict(json.loads(raw.decode()))
    except (ValueError, UnicodeDecodeError, TypeError):
        return EvalResult(stage="crash",
                          error=f"worker exited with code {proc.returncode} and no result "
                                f"(segfault or GPU fault?)\n{log.text()}",
                          duration_s=elapsed)
    if not res.compile_log:
        res.compile_log = log.text()
    res.duration_s = elapsed
    return res
