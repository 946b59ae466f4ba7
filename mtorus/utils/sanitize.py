"""Sanitizer builds of the host C++ runtime (race and memory-error detection).

The reference has no race detection (its only shared state is the mock mailbox
lock, crates/mt-comm/src/mock.rs:6-32).  Here the host library -- communicators,
fault plan, topology-aware wrapper, FP8 codec, pipeline schedules, token loader
(``csrc/comm``, ``csrc/core``, ``csrc/pipeline``) -- is plain C++17 with no
Python or CUDA dependency, so it can be compiled with a sanitizer into a native
stress driver (``csrc/tests/comm_stress.cpp``) that runs its thread-shared parts
from one thread per rank:

    python -m mtorus.utils.sanitize thread            # ThreadSanitizer
    python -m mtorus.utils.sanitize address           # AddressSanitizer + UBSan
    python -m mtorus.utils.sanitize thread --rounds 500

``run`` returns the driver's exit status and output; a sanitizer report makes the
status non-zero (``halt_on_error``).  Device code is not covered: the GPU kernels
check themselves (bounded waits, status words) instead.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile
from typing import Optional, Tuple

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
SOURCES = ["csrc/tests/comm_stress.cpp", "csrc/comm/comm.cpp", "csrc/comm/tcp.cpp", "csrc/comm/topology_aware.cpp",
           "csrc/core/topology.cpp", "csrc/core/precision.cpp", "csrc/core/data_loader.cpp",
           "csrc/pipeline/schedule.cpp"]
FLAGS = {
    "thread": ["-fsanitize=thread"],
    "address": ["-fsanitize=address,undefined", "-fno-omit-frame-pointer", "-fno-sanitize-recover=undefined"],
}
ENV = {
    "thread": {"TSAN_OPTIONS": "halt_on_error=1 exitcode=66 second_deadlock_stack=1"},
    "address": {"ASAN_OPTIONS": "halt_on_error=1 detect_leaks=1 exitcode=67",
                "UBSAN_OPTIONS": "halt_on_error=1 print_stacktrace=1"},
}


class SanitizerUnavailable(RuntimeError):
    """No compiler here can link the requested sanitizer's runtime library."""


def _compilers():
    """Candidate C++ compilers: MTORUS_SAN_CXX, then the system g++ / clang++, then $CXX
    (a toolchain installed for other builds may ship without the sanitizer runtimes)."""
    seen = []
    for c in (os.environ.get("MTORUS_SAN_CXX"), "g++", "clang++", os.environ.get("CXX")):
        path = shutil.which(c) if c else None
        if path and path not in seen:
            seen.append(path)
    return seen


def available() -> bool:
    return bool(_compilers())


def build(kind: str, out_dir: Optional[str] = None) -> str:
    """Compiles the stress driver with the ``kind`` sanitizer using the first compiler
    that can link its runtime; returns the binary path."""
    if kind not in FLAGS:
        raise ValueError(f"sanitizer kind must be one of {sorted(FLAGS)}")
    out_dir = out_dir or tempfile.mkdtemp(prefix="mtorus_san_")
    exe = os.path.join(out_dir, f"comm_stress_{kind}")
    errors = []
    for cxx in _compilers():
        cmd = [cxx, "-std=c++17", "-O1", "-g", *FLAGS[kind], "-I", os.path.join(ROOT, "csrc"),
               *[os.path.join(ROOT, s) for s in SOURCES], "-o", exe, "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode == 0:
            return exe
        errors.append(f"{cxx}: {r.stderr[-2000:]}")
    msg = "sanitizer build failed with every compiler:\n" + "\n".join(errors)
    if errors and all(("cannot find -l" in e and "san" in e) or "libtsan" in e or "libasan" in e for e in errors):
        raise SanitizerUnavailable(msg)
    raise RuntimeError(msg)


def run(kind: str, rounds: int = 50, timeout_s: float = 600.0, exe: Optional[str] = None) -> Tuple[int, str]:
    """Builds (unless ``exe`` is given) and runs the driver; returns (exit status, output)."""
    exe = exe or build(kind)
    env = dict(os.environ, **ENV[kind])
    r = subprocess.run([exe, str(int(rounds))], capture_output=True, text=True, timeout=timeout_s, env=env)
    return r.returncode, r.stdout + r.stderr


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("kind", choices=sorted(FLAGS))
    ap.add_argument("--rounds", type=int, default=50)
    args = ap.parse_args(argv)
    code, out = run(args.kind, args.rounds)
    sys.stdout.write(out)
    return code


if __name__ == "__main__":
    sys.exit(main())
