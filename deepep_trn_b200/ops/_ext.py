"""Loader of the compiled sm_100a extension ``deepep_trn_b200._C``.

The extension is built in-tree (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``). On a machine with a GPU a missing or broken
extension is an error, never a silent fallback to torch code.
"""
from __future__ import annotations

import importlib

_mod = None
_err: Exception | None = None


def load():
    global _mod, _err
    if _mod is not None:
        return _mod
    try:
        _mod = importlib.import_module('deepep_trn_b200._C')
    except Exception as exc:  # pragma: no cover - depends on the build
        _err = exc
        raise RuntimeError('deepep_trn_b200._C is not built: run `python setup.py build_ext --inplace` '
                           f'({type(exc).__name__}: {exc})') from exc
    return _mod


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False
