"""Loader for the compiled sm_100a extension (``dllm_qwen38_b200/_C*.so``).

The extension is built in-tree by ``setup.py build_ext --inplace`` (or ``__graft_entry__.build``)
and imported lazily, so CPU-only users never need it. On a CUDA tensor an op calls
``require()``, which raises with the import error instead of falling back.

``BDLLM_DEBUG_BOUNDS=1`` in the environment (read once, at the first load) selects the
debug-bounds build ``_C_dbg`` instead: the same kernels compiled with ``-DBDLLM_DEBUG_BOUNDS``,
which check indices, TMA coordinate alignment, vector-store alignment and epilogue values
(NaN / Inf sentinels) and record the first failure of each source file without trapping;
``bounds_report()`` returns those records.
"""

from __future__ import annotations

import importlib
import os

_STATE = {"mod": None, "err": None, "tried": False}


def module_name() -> str:
    return "_C_dbg" if os.environ.get("BDLLM_DEBUG_BOUNDS", "0") == "1" else "_C"


def _load():
    if not _STATE["tried"]:
        _STATE["tried"] = True
        try:
            _STATE["mod"] = importlib.import_module(f"..{module_name()}", __package__)
        except Exception as e:  # noqa: BLE001 - kept and re-raised by require()
            _STATE["err"] = f"{type(e).__name__}: {e}"
    return _STATE["mod"]


def available() -> bool:
    return _load() is not None


def bounds_report(reset: bool = True) -> list:
    """(file, line, index, limit, failures) for every source file whose checks failed since the
    last reset; always empty in the normal build."""
    return list(require().bounds_report(reset))


def require():
    if _load() is None:
        raise RuntimeError(
            "dllm_qwen38_b200 CUDA extension is not built or failed to load "
            f"({_STATE['err']}); run `python setup.py build_ext --inplace`"
        )
    return _STATE["mod"]


def __getattr__(name):
    # ops.<name> resolves to the autograd-aware wrapper in ops/cuda.py
    require()
    from . import cuda as _cuda

    try:
        return getattr(_cuda, name)
    except AttributeError:
        raise AttributeError(f"no native op {name!r}") from None
