"""Statement-by-statement sm_100a lowering for IRs no template accepts."""
from __future__ import annotations


class GenericLowering:
    name = "generic"

    def __init__(self, ctx):
        self.ctx = ctx

    def emit(self) -> str:
        raise NotImplementedError("no sm_100a template matches this kernel")
