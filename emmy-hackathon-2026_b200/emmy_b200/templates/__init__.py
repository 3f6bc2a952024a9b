"""Hand-written sm_100a kernel templates, tried in order by the compiler.

A template's module is imported the first time the compiler tries it, so a
one-kernel ``python compile.py`` loads only the templates it gets to (a
pointwise IR: the pointwise template alone).
"""
from __future__ import annotations

import importlib

from .common import TemplateMismatch


class _Lazy:
    """One registry entry: the template's ``name`` (what ``EMMY_TEMPLATE``
    selects) and its class, imported on first use."""

    def __init__(self, name: str, module: str, cls: str):
        self.name, self._module, self._cls, self._t = name, module, cls, None

    def load(self):
        if self._t is None:
            self._t = getattr(importlib.import_module(self._module, __name__), self._cls)
        return self._t

    def match(self, ctx):
        return self.load().match(ctx)


TEMPLATES = [_Lazy("pointwise", ".pointwise", "PointwiseTemplate"),
             _Lazy("rows", ".rows", "RowsTemplate"),
             _Lazy("gemm", ".gemm", "GemmTemplate"),
             _Lazy("gemm", ".gemm_small", "GemmSmallTemplate"),
             _Lazy("attention", ".attention", "AttentionTemplate"),
             _Lazy("attention", ".attention_small", "AttentionSmallTemplate")]

_CLASSES = {e._cls: e for e in TEMPLATES}


def __getattr__(name):
    """``from emmy_b200.templates import GemmTemplate`` and the like still
    work: the class is imported then."""
    if name in _CLASSES:
        return _CLASSES[name].load()
    raise AttributeError(name)


__all__ = ["TEMPLATES", "TemplateMismatch", "PointwiseTemplate", "RowsTemplate", "GemmTemplate",
           "AttentionTemplate", "GemmSmallTemplate", "AttentionSmallTemplate"]
