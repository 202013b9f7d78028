"""FSDP2 parameter all-gather and gradient reduce-scatter over NVLink peer memory.

The reference shards with FSDP2 and lets it run NCCL all-gather / reduce-scatter for
every block (ospnext/distributed/fsdp2_wrapper.py:11-77).  FSDP2 accepts custom
collectives per module (``set_custom_all_gather`` / ``set_custom_reduce_scatter``):
FSDP first asks the collective to ``allocate`` its buffer, copies this rank's part in,
then calls it.  Here those buffers are slots of one CUDA-IPC arena per rank, mapped by
every peer, and the collective is a tagged device barrier plus one pull kernel
(``ops/csrc/p2p.cu``):

* all-gather: each rank copies every peer's shard out of that peer's slot over NVLink;
* reduce-scatter (fp32 SUM / AVG): each rank sums its chunk of every peer's slot.  For
  modules whose FSDP ``param_dtype`` is bf16 (the transformer blocks) the slot holds the bf16
  gradients as autograd produced them and the pull kernel accumulates them in fp32: the
  bf16→fp32 cast that FSDP's copy-in would do is fused into the reduce-scatter (exact, since
  every bf16 value is an fp32 value) and half the bytes cross NVLink.

FSDP allocates these buffers in the same order on every rank, so the ring of slots
gives a slot the same offset everywhere; the barrier checks that (it carries the
offset as a tag) and the pull kernel does nothing if any peer disagrees or is late,
recording an error code that :func:`check` (and the trainers' per-step check) raises on.

Reusing a slot is ordered on the GPU, not only on the host.  Slot i of collective k is
written again by collective k + nslots (FSDP's copy-in, on its copy-in stream).  Before
that write the stream waits on two events of the slot:

* ``peers_done``: recorded on the collective's stream right after the barrier of
  collective k + 1 — every peer reaches that barrier only after its pull of collective k
  (same stream), so no peer still reads slot i;
* ``local_done``: recorded on the current stream when this rank drops its view of slot i
  (FSDP drops it right after enqueuing its copy-out on that stream), so this rank's own
  reads of the slot are ordered before the next write.

The IPC views are outside PyTorch's caching allocator, so these events replace its
stream tracking.  Anything the arena cannot hold (another dtype, a larger buffer) goes
to NCCL.
"""
from __future__ import annotations

import math
import weakref
from typing import List, Optional

import torch
import torch.distributed as dist
from torch.distributed.fsdp._fully_shard._fsdp_api import AllGather, ReduceScatter

from .. import ops


class _Arena:
    """One IPC segment per rank split into ``nslots`` equal slots, plus a flag array."""

    def __init__(self, group, slot_bytes: int, nslots: int, device, barrier_limit_s: float = 60.0):
        self.group = group
        self.barrier_limit_s = float(barrier_limit_s)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.slot_bytes = (int(slot_bytes) + 255) // 256 * 256
        self.nslots = nslots
        ext = ops.ext()
        self.base, h = ext.p2p_alloc(self.slot_bytes * nslots)
        self.flags, fh = ext.p2p_alloc(4 * (3 * self.world + 1))
        got = [None] * self.world
        dist.all_gather_object(got, (h, fh), group=group)
        self._opened: List[int] = []
        bases, flags = [], []
        for r in range(self.world):
            if r == self.rank:
                bases.append(self.base)
                flags.append(self.flags)
            else:
                b = ext.p2p_open(got[r][0])
                f = ext.p2p_open(got[r][1])
                self._opened += [b, f]
                bases.append(b)
                flags.append(f)
        self.bases = torch.tensor(bases, dtype=torch.int64, device=self.device)
        self.flag_ptrs = torch.tensor(flags, dtype=torch.int64, device=self.device)
        self.abort_ptr = self.flags + 4 * 3 * self.world
        self.next = 0
        self.epoch = 0
        self.live: List[Optional[weakref.ref]] = [None] * nslots
        self.peers_done: List[Optional[torch.cuda.Event]] = [None] * nslots
        self.local_done: List[Optional[torch.cuda.Event]] = [None] * nslots
        self._prev_slot: Optional[int] = None     # slot of the previous collective
        dist.barrier(group=group)

    def _record_local_done(self, i: int):
        def cb(_ref):
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self.local_done[i] = ev
        return cb

    def slot(self, numel: int, dtype: torch.dtype) -> Optional[torch.Tensor]:
        """The next slot as a ``numel`` view; the current stream (FSDP's copy-in stream)
        first waits until the slot's previous contents are no longer read anywhere."""
        nbytes = numel * torch.empty(0, dtype=dtype).element_size()
        if nbytes > self.slot_bytes:
            return None
        i = self.next
        prev = self.live[i]
        if prev is not None and prev() is not None:
            raise RuntimeError("P2P FSDP arena: slot still in use; raise nslots")
        self.next = (i + 1) % self.nslots
        stream = torch.cuda.current_stream(self.device)
        for evs in (self.peers_done, self.local_done):
            if evs[i] is not None:
                stream.wait_event(evs[i])
                evs[i] = None
        t = ops.ext().p2p_view(self.base + i * self.slot_bytes, [numel], dtype, self.device.index)
        self.live[i] = weakref.ref(t, self._record_local_done(i))
        return t

    def offset(self, t: torch.Tensor) -> Optional[int]:
        off = t.data_ptr() - self.base
        return off if 0 <= off < self.slot_bytes * self.nslots else None

    def barrier(self, tag: int, limit_s: Optional[float] = None):
        """Tagged device barrier on the current stream; afterwards no peer reads the slot of
        the previous collective any more (peers pull before they reach this barrier)."""
        self.epoch += 1
        limit = self.barrier_limit_s if limit_s is None else float(limit_s)
        ops.ext().p2p_barrier_tagged(self.flag_ptrs, self.rank, self.world, self.epoch, int(tag), limit)
        if self._prev_slot is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self.peers_done[self._prev_slot] = ev
        self._prev_slot = int(tag) // self.slot_bytes

    def close(self):
        """Unmap the peers' segments, wait for every rank to do the same, free our own."""
        ext = ops.ext()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            ext.p2p_close(p)
        self._opened = []
        dist.barrier(group=self.group)
        if self.base:
            ext.p2p_free(self.base)
            ext.p2p_free(self.flags)
            self.base = self.flags = 0


class P2PAllGather(AllGather):
    def __init__(self, arena: _Arena):
        self.arena = arena

    def allocate(self, size, *, dtype, device):
        t = self.arena.slot(math.prod(int(s) for s in size), dtype)
        return t.view(*size) if t is not None else torch.empty(*size, dtype=dtype, device=device)

    def __call__(self, output_tensor, input_tensor, group, async_op=False):
        off = self.arena.offset(output_tensor)
        if off is None:
            return dist.all_gather_into_tensor(output_tensor, input_tensor, group=group, async_op=async_op)
        shard_bytes = input_tensor.numel() * input_tensor.element_size()
        a = self.arena
        a.barrier(off)
        ops.ext().p2p_gather(a.bases, off, shard_bytes, a.rank, a.world, a.abort_ptr)
        return None


class P2PReduceScatter(ReduceScatter):
    """fp32 SUM / AVG; FSDP allocates the input (world × shard, in the arena) and then the
    output (shard, ordinary memory), in that order.  With ``grad_dtype=torch.bfloat16`` (the
    module's FSDP param_dtype, so its gradients arrive in bf16) the input slot is bf16: FSDP's
    copy-in then only copies, and the pull kernel sums the bf16 chunks in fp32 into the fp32
    output that FSDP asked for."""

    def __init__(self, arena: _Arena, grad_dtype: torch.dtype = torch.float32):
        self.arena = arena
        self.grad_dtype = grad_dtype
        self._want_input = True

    def allocate(self, size, *, dtype, device):
        numel = math.prod(int(s) for s in size)
        if self._want_input:
            self._want_input = False
            t = None
            if dtype == torch.float32:
                t = self.arena.slot(numel, torch.bfloat16 if self.grad_dtype == torch.bfloat16 else dtype)
            return t if t is not None else torch.empty(numel, dtype=dtype, device=device)
        self._want_input = True
        return torch.empty(numel, dtype=dtype, device=device)

    def __call__(self, output_tensor, input_tensor, group, op, async_op=False):
        off = self.arena.offset(input_tensor)
        scale = {dist.ReduceOp.SUM: 1.0, dist.ReduceOp.AVG: 1.0 / self.arena.world}.get(op)
        if off is None or scale is None or input_tensor.dtype not in (torch.float32, torch.bfloat16):
            if input_tensor.dtype != output_tensor.dtype:
                input_tensor = input_tensor.to(output_tensor.dtype)
            return dist.reduce_scatter_tensor(output_tensor, input_tensor, op=op, group=group, async_op=async_op)
        a = self.arena
        a.barrier(off)
        pull = (ops.ext().p2p_reduce_scatter_bf16 if input_tensor.dtype == torch.bfloat16
                else ops.ext().p2p_reduce_scatter_f32)
        pull(output_tensor, a.bases, off, output_tensor.numel(), a.rank, a.world, scale, a.abort_ptr)
        return None


def _group_shard_numel(module) -> int:
    state = module._get_fsdp_state()
    pg = state._fsdp_param_group
    return sum(fp.padded_sharded_param_size.numel() for fp in pg.fsdp_params) if pg is not None else 0


def _param_dtype(module) -> torch.dtype:
    """The FSDP2 mixed-precision param_dtype of a module (its gradients' dtype); fp32 when
    the module has no policy or the state cannot be read."""
    try:
        pol = module._get_fsdp_state()._mp_policy
        return pol.param_dtype or torch.float32
    except Exception:
        return torch.float32


def enable_p2p_fsdp(modules, group=None, nslots: int = 4, device=None, barrier_limit_s: float = 60.0):
    """Route the parameter all-gather and gradient reduce-scatter of the given FSDP2
    modules (the transformer blocks) through the NVLink pull kernels.  All modules share
    one all-gather arena and one reduce-scatter arena sized for the largest of them; modules
    with bf16 parameters reduce-scatter their bf16 gradients with fp32 accumulation.
    ``barrier_limit_s`` bounds each device barrier (a peer slower than that, e.g. stalled in
    data loading, makes the collective give up and record an error that the trainer's
    per-step check raises).  Returns the two arenas (call :func:`close` on them at exit)."""
    group = group or dist.group.WORLD
    world = dist.get_world_size(group)
    mods = [m for m in modules if hasattr(m, "set_custom_all_gather")]
    if world < 2 or not mods:
        return None
    n = max(_group_shard_numel(m) for m in mods)
    dev = device or torch.device("cuda", torch.cuda.current_device())
    grad_dtypes = [torch.bfloat16 if _param_dtype(m) == torch.bfloat16 else torch.float32 for m in mods]
    gbytes = 2 if all(d == torch.bfloat16 for d in grad_dtypes) else 4
    ag = _Arena(group, n * world * 2, nslots, dev, barrier_limit_s)        # bf16 parameters
    rs = _Arena(group, n * world * gbytes, nslots, dev, barrier_limit_s)   # bf16 or fp32 gradients
    rs.grad_bytes = gbytes
    for m, gd in zip(mods, grad_dtypes):
        m.set_custom_all_gather(P2PAllGather(ag))
        m.set_custom_reduce_scatter(P2PReduceScatter(rs, grad_dtype=gd))
    return ag, rs


def check(arenas, device_index: int):
    """Raise if a P2P collective timed out or saw mismatched slot offsets."""
    code = ops.ext().get_error(device_index, True)
    if code:
        raise RuntimeError(f"P2P FSDP collective failed on the device (error code {code})")


def close(arenas):
    if arenas:
        for a in arenas:
            a.close()
