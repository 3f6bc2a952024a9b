"""What a template or the generic lowering knows about one kernel: the IR
node, its launch descriptor (``meta.json``) and the graph's tensors.

Field meanings follow the reference compiler's constructor
(``compile.py:2285-2320``): the entry is the KernelOp's ``name`` (falling back
to meta's ``entry``), parameters are meta ``arg_order`` (``scalar: true``
arguments by value, everything else a ``.u64`` pointer), and grid/block/
``smem_bytes`` come from the meta kernel whose ``entry`` matches.
"""
from __future__ import annotations

from math import prod

from .analysis import Buffers, kind
from .ir import dim
from .ptx import PARAM_TYPES


class KernelContext:
    def __init__(self, graph, meta: dict, node_name: str):
        self.graph = graph
        self.meta = meta
        self.node_name = node_name
        self.op = graph.nodes[node_name].op
        self.entry = self.op.name or (meta["kernels"][0].get("entry") if meta.get("kernels") else None) \
            or node_name
        self.bufs = Buffers()
        for nd in graph.nodes.values():
            for t in nd.outputs:
                self.bufs.shapes[t.name] = tuple(dim(d) for d in t.shape)
                self.bufs.dtypes[t.name] = getattr(t.dtype, "name", t.dtype)
            if type(nd.op).__name__ == "ConstantOp":
                self.bufs.constants[nd.name] = getattr(nd.op, "value", None)
        kernels = meta.get("kernels") or []
        info = next((k for k in kernels if k.get("entry") == self.entry), None)
        if info is None:
            if not kernels:
                raise ValueError("meta.json has no kernels")
            info = kernels[0]
        self.info = info
        # the launch descriptor's argument dtypes are what the runtime
        # allocates; where the graph's tensor dtype disagrees (an IR whose
        # writes convert, e.g. f32 arithmetic stored to an i32 buffer), the
        # buffer's own dtype wins
        for a in info.get("args", []):
            if not a.get("scalar") and a.get("dtype") and a["name"] in self.bufs.dtypes:
                self.bufs.dtypes[a["name"]] = a["dtype"]
        self.arg_order = list(info["arg_order"])
        self.scalar_tys = {a["name"]: a["dtype"] for a in info.get("args", []) if a.get("scalar")}
        self.grid = tuple(int(x) for x in info["grid"])
        self.block = tuple(int(x) for x in info["block"])
        self.smem_bytes = int(info.get("smem_bytes", 0) or 0)
        self.zero_outputs = list(info.get("zero_outputs", []) or [])
        self.outputs = [nd.outputs[0].name for nd in [graph.nodes[node_name]]]
        body = self.op.body
        self.tile = body[0] if len(body) == 1 and kind(body[0]) == "Tile" else None

    @property
    def threads(self) -> int:
        return prod(self.block)

    @property
    def total_threads(self) -> int:
        return prod(self.grid) * prod(self.block)

    def params(self) -> list:
        out = []
        for a in self.arg_order:
            if a in self.scalar_tys:
                out.append((a, PARAM_TYPES.get(self.scalar_tys[a], "u32")))
            else:
                out.append((a, "u64"))
        return out

    def tile_axes(self) -> list:
        return [(a.name, dim(a.extent)) for a in self.tile.axes]
