"""Cross-GPU finish of the global sum over NVLink peer memory.

The path's one cross-GPU reduction is the global sum: every rank's sum kernel
leaves a partial ``f32[1]``.  :func:`dist.global_sum` finishes it with an NCCL
all-reduce; :class:`PeerSum` finishes it without a collective library, in one
single-thread kernel per rank:

* at set-up every rank allocates a slot array (two sets of one 128-byte
  slot per rank, then an epoch word) with ``emmy_mem_alloc``, exports it
  (``emmy_ipc_handle``), gathers the other ranks' handles through the process
  group and maps their arrays (``emmy_ipc_open``: CUDA IPC, peer access over
  NVLink enabled as needed -- plain peer stores, no multicast object);
* the kernel (``emmy_peer_sum``) reads this rank's partial, packs it with the
  launch's epoch into one 64-bit word and stores that word into its own slot
  of every rank's array (``st.release.sys``, one NVLink write per peer); then
  it polls its own array (``ld.acquire.sys``) until every rank's word carries
  this epoch, sums the values in rank order -- the same order on every rank,
  so every rank gets the same bits -- writes the sum over the partial and
  advances the epoch word;
* the slot set alternates with the epoch's parity: a rank can start writing
  epoch e+2 only after its launch e+1 saw every rank's epoch-e+1 word, which
  every rank writes after its launch e completed -- so no word is
  overwritten before every rank has read it;
* the epoch lives in device memory, so the launch can be replayed from a CUDA
  graph; every rank launches the kernel the same number of times;
* each poll is bounded by ``%globaltimer`` (2 s): on expiry the kernel stores
  code 9 in the module's ``__emmy_status`` word and returns, leaving the
  partial and the epoch as they were.

The same exchange also runs inside the split full-sum kernel itself
(:func:`emit_fused_finish`, the kernel's last CTA): one kernel per rank does
the sum and the cross-GPU finish.

The kernels of different ranks wait on one another, so they must run on
different GPUs at the same time: one process per GPU, as the benchmark runs.
"""
from __future__ import annotations

import ctypes

from . import native

SLOT = 128                     # bytes per rank's slot (one cache line each)
WAIT_NS = 2_000_000_000        # bound of every poll: 2 s of %globaltimer
STATUS_TIMEOUT = 9

PEER_SUM_PTX = f"""\
.version 8.8
.target sm_100a
.address_size 64

.global .align 4 .u32 __emmy_status;

.visible .entry emmy_peer_sum(.param .u64 p_sum, .param .u64 p_peers, .param .u64 p_local,
                              .param .u32 p_rank, .param .u32 p_world)
{{
  .reg .pred %p<6>;
  .reg .b32 %r<12>;
  .reg .b64 %rd<16>;
  .reg .f32 %f<4>;
  mov.u32 %r0, %tid.x;
  setp.ne.u32 %p0, %r0, 0;
  @%p0 bra DONE;
  ld.param.u64 %rd0, [p_sum];
  ld.param.u64 %rd1, [p_peers];
  ld.param.u64 %rd2, [p_local];
  ld.param.u32 %r1, [p_rank];
  ld.param.u32 %r2, [p_world];
  // this launch's epoch: the local epoch word (after both slot sets) + 1
  mul.wide.u32 %rd3, %r2, {2 * SLOT};
  add.s64 %rd4, %rd2, %rd3;
  ld.global.u32 %r3, [%rd4];
  add.u32 %r3, %r3, 1;
  // the epoch's slot set: (epoch & 1) * world slots in
  and.b32 %r8, %r3, 1;
  mul.lo.u32 %r8, %r8, %r2;
  // this rank's partial and epoch in one 64-bit word (value low, epoch high)
  ld.global.f32 %f0, [%rd0];
  mov.b32 %r4, %f0;
  mov.b64 %rd5, {{%r4, %r3}};
  add.u32 %r9, %r8, %r1;
  mul.wide.u32 %rd6, %r9, {SLOT};
  mov.u32 %r5, 0;
PUT:
  mul.wide.u32 %rd7, %r5, 8;
  add.s64 %rd7, %rd1, %rd7;
  ld.global.u64 %rd8, [%rd7];
  add.s64 %rd8, %rd8, %rd6;
  st.release.sys.global.u64 [%rd8], %rd5;
  add.u32 %r5, %r5, 1;
  setp.lt.u32 %p1, %r5, %r2;
  @%p1 bra PUT;
  // every rank's word of this epoch, summed in rank order
  mov.f32 %f1, 0f00000000;
  mov.u64 %rd9, %globaltimer;
  mov.u32 %r5, 0;
GET:
  add.u32 %r10, %r8, %r5;
  mul.wide.u32 %rd10, %r10, {SLOT};
  add.s64 %rd10, %rd2, %rd10;
SPIN:
  ld.acquire.sys.global.u64 %rd11, [%rd10];
  mov.b64 {{%r6, %r7}}, %rd11;
  setp.eq.u32 %p2, %r7, %r3;
  @%p2 bra GOT;
  mov.u64 %rd12, %globaltimer;
  sub.s64 %rd12, %rd12, %rd9;
  setp.lt.s64 %p3, %rd12, {WAIT_NS};
  @%p3 bra SPIN;
  st.global.u32 [__emmy_status], {STATUS_TIMEOUT};
  bra DONE;
GOT:
  mov.b32 %f2, %r6;
  add.rn.f32 %f1, %f1, %f2;
  add.u32 %r5, %r5, 1;
  setp.lt.u32 %p4, %r5, %r2;
  @%p4 bra GET;
  st.global.f32 [%rd0], %f1;
  st.global.u32 [%rd4], %r3;
DONE:
  ret;
}}
"""


# the fused form: a full-sum kernel compiled with ``"peer_finish": true`` in
# its meta launch descriptor takes these four parameters after meta
# arg_order (``// @emmy peer`` in its PTX) and finishes the global sum itself
FUSED_PARAMS = [("peer_table", "u64"), ("peer_local", "u64"), ("peer_rank", "u32"),
                ("peer_world", "u32")]


def emit_fused_finish(k, sum_addr: str, ncta: int, status: str, done_sym: str) -> None:
    """The cross-GPU finish inside the split full-sum kernel itself, emitted
    after thread 0 of a CTA has added the CTA's partial into ``sum_addr`` (a
    global address register): one acquire-release atomic on the module's
    completion counter ``done_sym`` finds the launch's last CTA, which reads
    the rank's complete partial, resets
    the counter for the next launch, and runs the exchange of the
    single-thread ``emmy_peer_sum`` kernel -- its partial packed with the
    epoch into every rank's slot (``st.release.sys``), its own slots polled
    (``ld.acquire.sys``, bounded by ``WAIT_NS``; ``STATUS_TIMEOUT`` into
    ``status`` on expiry) and summed in rank order over ``sum_addr``.  The
    other CTAs leave as soon as they have counted themselves, so the partial
    is final when the exchange starts and no CTA waits on another GPU but
    the last."""
    done = k.label("PEER_DONE")
    old = k.reg("r")
    # the count is an acquire-release RMW: it publishes this CTA's partial
    # (added just before) and, in the last CTA, sees every other CTA's
    k(f"atom.acq_rel.gpu.global.add.u32 {old}, [{done_sym}], 1;")
    p = k.reg("p")
    k(f"setp.ne.u32 {p}, {old}, {ncta - 1};")
    k(f"@{p} bra {done};")
    part = k.reg("f")
    k(f"ld.relaxed.gpu.global.f32 {part}, [{sum_addr}];")
    k(f"st.relaxed.gpu.global.u32 [{done_sym}], 0;")
    peers, local = k.reg("rd"), k.reg("rd")
    rank, world = k.reg("r"), k.reg("r")
    k(f"ld.param.u64 {peers}, [param_peer_table];")
    k(f"ld.param.u64 {local}, [param_peer_local];")
    k(f"ld.param.u32 {rank}, [param_peer_rank];")
    k(f"ld.param.u32 {world}, [param_peer_world];")
    # this launch's epoch: the local epoch word (after both slot sets) + 1
    eoff = k.reg("rd")
    k(f"mul.wide.u32 {eoff}, {world}, {2 * SLOT};")
    eaddr = k.reg("rd")
    k(f"add.s64 {eaddr}, {local}, {eoff};")
    ep = k.reg("r")
    k(f"ld.global.u32 {ep}, [{eaddr}];")
    k(f"add.u32 {ep}, {ep}, 1;")
    # the epoch's slot set, this rank's word (value low, epoch high)
    set0 = k.reg("r")
    k(f"and.b32 {set0}, {ep}, 1;")
    k(f"mul.lo.u32 {set0}, {set0}, {world};")
    vb = k.reg("r")
    k(f"mov.b32 {vb}, {part};")
    word = k.reg("rd")
    k(f"mov.b64 {word}, {{{vb}, {ep}}};")
    mine = k.reg("r")
    k(f"add.u32 {mine}, {set0}, {rank};")
    moff = k.reg("rd")
    k(f"mul.wide.u32 {moff}, {mine}, {SLOT};")
    i = k.reg("r")
    k(f"mov.u32 {i}, 0;")
    put = k.label("PEER_PUT")
    k.mark(put)
    pa = k.reg("rd")
    k(f"mul.wide.u32 {pa}, {i}, 8;")
    k(f"add.s64 {pa}, {peers}, {pa};")
    base = k.reg("rd")
    k(f"ld.global.u64 {base}, [{pa}];")
    dst = k.reg("rd")
    k(f"add.s64 {dst}, {base}, {moff};")
    k(f"st.release.sys.global.u64 [{dst}], {word};")
    k(f"add.u32 {i}, {i}, 1;")
    pl = k.reg("p")
    k(f"setp.lt.u32 {pl}, {i}, {world};")
    k(f"@{pl} bra {put};")
    # every rank's word of this epoch, summed in rank order
    acc = k.reg("f")
    k(f"mov.f32 {acc}, 0f00000000;")
    t0 = k.reg("rd")
    k(f"mov.u64 {t0}, %globaltimer;")
    k(f"mov.u32 {i}, 0;")
    get, spin, got = k.label("PEER_GET"), k.label("PEER_SPIN"), k.label("PEER_GOT")
    k.mark(get)
    sl = k.reg("r")
    k(f"add.u32 {sl}, {set0}, {i};")
    sa = k.reg("rd")
    k(f"mul.wide.u32 {sa}, {sl}, {SLOT};")
    k(f"add.s64 {sa}, {local}, {sa};")
    k.mark(spin)
    w = k.reg("rd")
    k(f"ld.acquire.sys.global.u64 {w}, [{sa}];")
    lo, hi = k.reg("r"), k.reg("r")
    k(f"mov.b64 {{{lo}, {hi}}}, {w};")
    pe = k.reg("p")
    k(f"setp.eq.u32 {pe}, {hi}, {ep};")
    k(f"@{pe} bra {got};")
    t1 = k.reg("rd")
    k(f"mov.u64 {t1}, %globaltimer;")
    k(f"sub.s64 {t1}, {t1}, {t0};")
    pt = k.reg("p")
    k(f"setp.lt.s64 {pt}, {t1}, {WAIT_NS};")
    k(f"@{pt} bra {spin};")
    k(f"st.global.u32 [{status}], {STATUS_TIMEOUT};")
    k(f"bra {done};")
    k.mark(got)
    v = k.reg("f")
    k(f"mov.b32 {v}, {lo};")
    k(f"add.rn.f32 {acc}, {acc}, {v};")
    k(f"add.u32 {i}, {i}, 1;")
    pg = k.reg("p")
    k(f"setp.lt.u32 {pg}, {i}, {world};")
    k(f"@{pg} bra {get};")
    k(f"st.global.f32 [{sum_addr}], {acc};")
    k(f"st.global.u32 [{eaddr}], {ep};")
    k.mark(done)


def exchange_handles(handle: bytes, world: int) -> list:
    """Every rank's 64-byte handle, in rank order (through the process
    group; a one-process job has only its own)."""
    if world <= 1:
        return [handle]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, handle)
    return out


class PeerSum:
    """The cross-GPU sum of one ``f32`` per rank, finished over NVLink peer
    memory (see the module docstring).  ``launch(sum_ptr, stream)`` replaces
    the rank's partial at ``sum_ptr`` by the sum of every rank's partial."""

    def __init__(self, rank: int, world: int):
        L = native.lib()
        self.rank, self.world = rank, world
        self.nbytes = (2 * world + 1) * SLOT
        p = ctypes.c_uint64()
        self.local = self.peer_table = 0
        self.peers = []
        # every rank joins the exchange, with None if its own export failed,
        # so that all ranks fail together instead of waiting for each other
        mine = None
        try:
            native.check(L.emmy_mem_alloc(ctypes.byref(p), self.nbytes))
            self.local = p.value
            native.check(L.emmy_memset_async(self.local, 0, self.nbytes, None))
            native.check(L.emmy_stream_sync(None))
            buf = ctypes.create_string_buffer(64)
            native.check(L.emmy_ipc_handle(self.local, buf))
            mine = buf.raw
        except native.EmmyError:
            pass
        handles = exchange_handles(mine, world)
        if any(h is None for h in handles):
            if self.local:
                native.check(L.emmy_mem_free(self.local))
            raise RuntimeError("a rank could not export its peer-sum slots")
        for r, h in enumerate(handles):
            if r == rank:
                self.peers.append(self.local)
                continue
            q = ctypes.c_uint64()
            native.check(L.emmy_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(q)))
            self.peers.append(q.value)
        arr = (ctypes.c_uint64 * world)(*self.peers)
        native.check(L.emmy_mem_alloc(ctypes.byref(p), 8 * world))
        self.peer_table = p.value
        native.check(L.emmy_memcpy_htod_async(self.peer_table, ctypes.addressof(arr), 8 * world,
                                              None))
        native.check(L.emmy_stream_sync(None))
        self.image = native.Image(PEER_SUM_PTX)
        self.module = native.Module(self.image.data)
        self.kernel = self.module.kernel("emmy_peer_sum")

    def status(self) -> int:
        """The module's status word (0, or 9 after a poll that timed out)."""
        L = native.lib()
        addr, _ = self.module.global_addr("__emmy_status")
        v = ctypes.c_uint32()
        native.check(L.emmy_memcpy_dtoh_async(ctypes.addressof(v), addr, 4, None))
        native.check(L.emmy_stream_sync(None))
        return v.value

    def fused_values(self) -> dict:
        """The values of ``FUSED_PARAMS`` for a fused full-sum kernel's launch
        (keyed by parameter name, as ``harness.CompiledKernel.params`` takes
        them beside the meta arguments)."""
        return {"peer_table": self.peer_table, "peer_local": self.local,
                "peer_rank": self.rank, "peer_world": self.world}

    def launch(self, sum_ptr: int, stream) -> None:
        L = native.lib()
        args = [ctypes.c_uint64(sum_ptr), ctypes.c_uint64(self.peer_table),
                ctypes.c_uint64(self.local), ctypes.c_uint32(self.rank),
                ctypes.c_uint32(self.world)]
        params = (ctypes.c_void_p * len(args))(*[ctypes.addressof(a) for a in args])
        native.check(L.emmy_launch(self.kernel.h, native.u32x3((1, 1, 1)),
                                   native.u32x3((32, 1, 1)), 0, None, params, stream))

    def close(self, barrier=None) -> None:
        """Unmap the peers' arrays, then free this rank's own (every rank's
        kernels must have completed).  ``barrier`` (the process group's)
        runs between the two, so no rank frees an array another rank still
        has mapped."""
        L = native.lib()
        for r, q in enumerate(self.peers):
            if r != self.rank and q:
                native.check(L.emmy_ipc_close(q))
        self.peers = []
        if barrier is not None:
            barrier()
        for a in ("peer_table", "local"):
            if getattr(self, a, 0):
                native.check(L.emmy_mem_free(getattr(self, a)))
                setattr(self, a, 0)
        self.module.unload()
