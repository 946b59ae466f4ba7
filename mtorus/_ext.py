"""Loader for the in-tree compiled extensions.

``mtorus._C`` is the host C++ runtime and ``mtorus._cuda`` the sm_100a kernels.
Both are built in place by ``python setup.py build_ext --inplace``.  On a
machine with a GPU a missing kernel extension is an error: there is no silent
eager fallback for the fused kernels.
"""
from __future__ import annotations

import importlib
import os
import subprocess
import sys
import threading

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_lock = threading.Lock()
_mods: dict = {}


def build_inplace(quiet: bool = True) -> None:
    """Compile both extensions in the source tree (ninja, incremental)."""
    env = dict(os.environ)
    env.setdefault("MAX_JOBS", str(max(1, min(16, os.cpu_count() or 1))))
    cmd = [sys.executable, "setup.py", "build_ext", "--inplace"]
    out = subprocess.run(cmd, cwd=_ROOT, env=env, capture_output=quiet, text=True)
    if out.returncode != 0:
        msg = (out.stdout or "")[-4000:] + (out.stderr or "")[-4000:] if quiet else ""
        raise RuntimeError(f"mtorus extension build failed:\n{msg}")


def _load(name: str):
    with _lock:
        if name in _mods:
            return _mods[name]
        import torch  # noqa: F401  (loads libtorch before the extension)

        try:
            mod = importlib.import_module(f"mtorus.{name}")
        except ImportError:
            if os.environ.get("MTORUS_NO_AUTOBUILD"):
                raise
            build_inplace()
            mod = importlib.import_module(f"mtorus.{name}")
        _mods[name] = mod
        return mod


def host():
    """The host C++ runtime module (topology, FP8 codec, communicators, schedules)."""
    return _load("_C")


def cuda():
    """The sm_100a kernel module."""
    return _load("_cuda")


def cuda_available() -> bool:
    import torch

    return torch.cuda.is_available()
