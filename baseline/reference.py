"""Loader of the reference's own code, installed under ``baseline/_ref``.

``baseline/_ref`` holds the unmodified NebulaSD packages (``swiftllm`` and
``nebulasd``), installed from the reference checkout with

    python -m pip install --no-index --no-build-isolation --no-deps \\
        --find-links /opt/wheelhouse --target baseline/_ref <copy>/swiftLLM <copy>/nebulasd

(built from a copy under /tmp because the checkout is read-only).  The
directory is git-ignored but travels with the repository to the GPU box, where
it serves three purposes: the reference's Triton kernels JIT-compiled on the
same B200 as the bar in ``bench.py``, the reference's ``LlamaModel`` as the
accept-identity check, and the reference's HostKV arena / copy executor as
the real objects ``NativeCopyBackend`` is dropped into.  Nothing in the
product (``nebulasd_b200``) imports this module.

``swiftllm/__init__.py`` imports the serving stack (``ray`` and the compiled
``swiftllm_c`` extension), which the kernels and the model do not use, so the
package is mounted as a namespace module and ``swiftllm_c`` gets an empty
stand-in (only ``LlamaModel._swap``, CPU swapping, calls it).
"""
from __future__ import annotations

import importlib
import sys
import types
from pathlib import Path

REF = Path(__file__).resolve().parent / "_ref"


def available() -> bool:
    """True when the reference packages are installed under ``baseline/_ref``."""
    return (REF / "swiftllm" / "worker" / "kernels" / "paged_attn.py").exists() and \
        (REF / "nebulasd" / "kv" / "arena.py").exists()


def _mount() -> None:
    if not available():
        raise ImportError(f"the reference is not installed under {REF}")
    mod = sys.modules.get("swiftllm")
    if mod is None or list(getattr(mod, "__path__", [])) != [str(REF / "swiftllm")]:
        mod = types.ModuleType("swiftllm")
        mod.__path__ = [str(REF / "swiftllm")]
        sys.modules["swiftllm"] = mod
    if "swiftllm_c" not in sys.modules:
        sys.modules["swiftllm_c"] = types.ModuleType("swiftllm_c")
    if str(REF) not in sys.path:
        sys.path.append(str(REF))


def swiftllm(name: str):
    """Import ``swiftllm.<name>`` from the installed reference (e.g. ``worker.kernels.paged_attn``)."""
    _mount()
    return importlib.import_module(f"swiftllm.{name}")


def nebulasd(name: str):
    """Import ``nebulasd.<name>`` from the installed reference (e.g. ``kv.arena``)."""
    _mount()
    return importlib.import_module(f"nebulasd.{name}")
