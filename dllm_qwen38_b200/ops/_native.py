"""Loader for the compiled sm_100a extension (``dllm_qwen38_b200/_C*.so``).

The extension is built in-tree by ``setup.py build_ext --inplace`` (or ``__graft_entry__.build``)
and imported lazily, so CPU-only users never need it. On a CUDA tensor an op calls
``require()``, which raises with the import error instead of falling back.
"""

from __future__ import annotations

_STATE = {"mod": None, "err": None, "tried": False}


def _load():
    if not _STATE["tried"]:
        _STATE["tried"] = True
        try:
            from .. import _C  # noqa: F401

            _STATE["mod"] = _C
        except Exception as e:  # noqa: BLE001 - kept and re-raised by require()
            _STATE["err"] = f"{type(e).__name__}: {e}"
    return _STATE["mod"]


def available() -> bool:
    return _load() is not None


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
