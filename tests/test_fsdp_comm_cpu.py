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
