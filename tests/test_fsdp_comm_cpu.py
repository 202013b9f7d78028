"""Host-side logic of the NVLink FSDP collectives (slot ring, allocation order, fallbacks)
with a fake arena; the device kernels are covered by tests/test_multigpu.py."""
import weakref

import pytest
import torch

from osp_next_b200.parallel import fsdp_comm


class FakeArena:
    def __init__(self, slot_bytes=1024, nslots=2):
        self.slot_bytes, self.nslots, self.world, self.rank = slot_bytes, nslots, 2, 0
        self.mem = torch.zeros(slot_bytes * nslots, dtype=torch.uint8)
        self.base = self.mem.data_ptr()
        self.next = 0
        self.live = [None] * nslots
        self.calls = []

    def slot(self, numel, dtype):
        nbytes = numel * torch.empty(0, dtype=dtype).element_size()
        if nbytes > self.slot_bytes:
            return None
        i = self.next
        if self.live[i] is not None and self.live[i]() is not None:
            raise RuntimeError("slot still in use")
        self.next = (i + 1) % self.nslots
        t = self.mem[i * self.slot_bytes:i * self.slot_bytes + nbytes].view(dtype)
        self.live[i] = weakref.ref(t)
        return t

    def offset(self, t):
        off = t.data_ptr() - self.base
        return off if 0 <= off < self.slot_bytes * self.nslots else None


def test_reduce_scatter_allocates_input_in_arena_then_output_outside():
    a = FakeArena()
    rs = fsdp_comm.P2PReduceScatter(a)
    inp = rs.allocate((64,), dtype=torch.float32, device="cpu")
    out = rs.allocate((32,), dtype=torch.float32, device="cpu")
    assert a.offset(inp) == 0 and a.offset(out) is None
    inp2 = rs.allocate((64,), dtype=torch.float32, device="cpu")
    assert a.offset(inp2) == a.slot_bytes          # next slot of the ring
    rs.allocate((32,), dtype=torch.float32, device="cpu")
    # bf16 gradients are not handled by the fp32 pull kernel: ordinary memory, NCCL later
    x = rs.allocate((64,), dtype=torch.bfloat16, device="cpu")
    assert a.offset(x) is None


def test_reduce_scatter_bf16_gradients_use_a_bf16_slot():
    # FSDP asks for an fp32 input (reduce_dtype); with bf16 gradients the slot is bf16, so
    # the copy-in only copies and the pull kernel does the fp32 accumulation
    a = FakeArena()
    rs = fsdp_comm.P2PReduceScatter(a, grad_dtype=torch.bfloat16)
    inp = rs.allocate((64,), dtype=torch.float32, device="cpu")
    out = rs.allocate((32,), dtype=torch.float32, device="cpu")
    assert inp.dtype == torch.bfloat16 and a.offset(inp) == 0
    assert out.dtype == torch.float32 and a.offset(out) is None
    # a non-fp32 reduce dtype never goes to the arena
    x = rs.allocate((64,), dtype=torch.bfloat16, device="cpu")
    assert a.offset(x) is None


def test_reduce_scatter_fallback_casts_bf16_input_for_nccl(monkeypatch):
    a = FakeArena()
    rs = fsdp_comm.P2PReduceScatter(a, grad_dtype=torch.bfloat16)
    seen = {}

    def fake_rs(out, inp, op=None, group=None, async_op=False):
        seen["dtype"] = inp.dtype
        out.copy_(inp[:out.numel()])

    monkeypatch.setattr(fsdp_comm.dist, "reduce_scatter_tensor", fake_rs)
    inp = torch.ones(64, dtype=torch.bfloat16)          # outside the arena → c10d path
    out = torch.zeros(32, dtype=torch.float32)
    rs(out, inp, group=None, op=fsdp_comm.dist.ReduceOp.SUM)
    assert seen["dtype"] == torch.float32 and torch.all(out == 1)


def test_param_dtype_reads_the_fsdp_policy():
    class Pol:
        param_dtype = torch.bfloat16

    class State:
        _mp_policy = Pol()

    class M:
        def _get_fsdp_state(self):
            return State()

    assert fsdp_comm._param_dtype(M()) == torch.bfloat16
    assert fsdp_comm._param_dtype(object()) == torch.float32


def test_all_gather_slot_ring_and_oversize_fallback():
    a = FakeArena(slot_bytes=256, nslots=2)
    ag = fsdp_comm.P2PAllGather(a)
    t0 = ag.allocate((64,), dtype=torch.bfloat16, device="cpu")
    t1 = ag.allocate((64,), dtype=torch.bfloat16, device="cpu")
    assert a.offset(t0) == 0 and a.offset(t1) == 256
    big = ag.allocate((1024,), dtype=torch.bfloat16, device="cpu")
    assert a.offset(big) is None                    # larger than a slot → NCCL path
    with pytest.raises(RuntimeError):               # slot 0 still referenced: never overwritten
        ag.allocate((64,), dtype=torch.bfloat16, device="cpu")
    del t0
    t2 = ag.allocate((64,), dtype=torch.bfloat16, device="cpu")
    assert a.offset(t2) == 0
