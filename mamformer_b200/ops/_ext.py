"""Loader for the in-tree native extension ``mamformer_b200._C`` (sm_100a kernels)."""

from __future__ import annotations

import importlib

_C = None
_ERR: Exception | None = None


def _load():
    global _C, _ERR
    if _C is not None or _ERR is not None:
        return
    try:
        _C = importlib.import_module("mamformer_b200._C")
    except Exception as e:  # ImportError or an undefined-symbol OSError
        _ERR = e


def ext():
    _load()
    return _C


def has_native() -> bool:
    _load()
    return _C is not None


def require_native():
    """Raise when a CUDA op is requested but the native extension is not importable."""
    _load()
    if _C is None:
        raise RuntimeError(
            "mamformer_b200 native extension (_C) is not available: build it with "
            "`python setup.py build_ext --inplace` (or __graft_entry__.build()). "
            f"Import error: {_ERR!r}")
    return _C


def bounds_errors() -> dict:
    """Read and clear the bounds-check error words of the native modules: ``{name: code}`` for
    every word that is set.  Only kernels compiled with MAMF_BOUNDS_CHECK record anything (the
    module ``_C_check`` always is; ``_C`` when built with MAMF_BOUNDS_CHECK=1)."""
    out = {}
    mods = [("_C", ext())]
    try:
        mods.append(("_C_check", importlib.import_module("mamformer_b200._C_check")))
    except Exception:
        pass
    for name, mod in mods:
        if mod is None:
            continue
        for fn in ("bounds_error_moe_rows", "bounds_error_ce"):
            v = int(getattr(mod, fn)())
            if v:
                out[f"{name}.{fn[len('bounds_error_'):]}"] = v
    return out
