"""Roofline benchmark of the fused SSP exchange (FFN-down GEMM + P2P row stores).

Run one process per GPU (``torchrun --nproc-per-node N -m benchmarks.ssp_exchange``).
At the 14B shapes (81f 768×1280 → grid 21×48×80, P = 2) each rank holds its Token-layout
rows; the FFN-down + gated-residual GEMM of that block writes every output row straight
into the rank that owns it in the next (Group) layout.  Timed, on every rank with CUDA
events after warm-up, max over ranks:

  local   the same GEMM with the residual epilogue storing locally (no exchange)
  p2p     the fused GEMM storing into the owners' buffers over NVLink + the flag barrier
  nccl    local GEMM, then the reference's exchange: gather rows by destination,
          ``all_to_all_single``, scatter into the Group layout

Roofline of the fused path = max(GEMM FLOPs ÷ measured bf16 peak, bytes that leave the
GPU ÷ 770 GB/s per direction); the line reports achieved = roofline ÷ p2p time.

The exchange alone (the training path, where autograd keeps the result) is timed too:

  staged       ``p2p_redistribute`` forward: stage the rows in peer memory, barrier, pull
               this rank's next-layout rows into a fresh tensor
  staged_bwd   its backward (gradient rows pulled back to their owners)
  nccl_xchg    gather rows by destination, ``all_to_all_single``, scatter

with roofline max(bytes that cross NVLink ÷ 770 GB/s, local HBM bytes ÷ measured copy
bandwidth): HBM traffic is the stage copy (read + write) plus the pull's local writes.
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

from osp_next_b200 import ops
from osp_next_b200.models.layout import GROUP, TOKEN, ParallelSpec, make_layout, make_redistribution
from osp_next_b200.parallel.p2p import P2PExchange

NVLINK_GBS = 770.0


def _peak_tflops() -> float:
    p = os.path.join(os.path.dirname(__file__), "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d.get("bf16_tflops") or d.get("bf16_tflops_sustained"))
    except Exception:
        return 1400.0


def _hbm_gbs() -> float:
    p = os.path.join(os.path.dirname(__file__), "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f).get("hbm_gbs"))
    except Exception:
        return 6650.0


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    grid, P, C, F = (21, 48, 80), 2, 5120, 13824
    spec = ParallelSpec(world, 1, world, rank)
    la = make_layout(TOKEN, grid, P, spec)
    lb = make_layout(GROUP, grid, P, spec)
    rd = make_redistribution(TOKEN, GROUP, grid, P, spec)
    n = la.n_local
    torch.manual_seed(rank)
    h = torch.randn(1, n, F, device=dev).to(torch.bfloat16)
    w = (torch.randn(C, F, device=dev) / F ** 0.5).to(torch.bfloat16)
    b = torch.randn(C, device=dev)
    gate = torch.randn(1, C, device=dev)
    resid = torch.randn(1, n, C, device=dev)
    n_stride = max(make_layout(k, grid, P, ParallelSpec(world, 1, world, r)).n_local
                   for k in (TOKEN, GROUP) for r in range(world))
    ex = P2PExchange(dist.group.WORLD, 1, n_stride, C, dev)
    drank = rd.dest_rank.to(dev, torch.int32)
    drow = rd.dest_row.to(dev, torch.int32)
    out_local = torch.empty(1, n, C, device=dev)

    def run_local():
        ops.linear_gated_residual(h, w, b, resid, gate, out=out_local)

    def run_p2p():
        ops.linear_gated_residual_p2p(h, w, b, resid, gate, drank, drow, ex.target(), n_stride)
        ex.barrier()
        ex.take(lb.n_local)

    send_rows = rd.send_rows.to(dev)
    recv_rows = rd.recv_rows.to(dev)
    recv_buf = torch.empty(1, lb.n_local, C, device=dev)

    def run_nccl():
        ops.linear_gated_residual(h, w, b, resid, gate, out=out_local)
        send = out_local[0].index_select(0, send_rows)
        recv = torch.empty(int(sum(rd.recv_counts)), C, device=dev)
        dist.all_to_all_single(recv, send, rd.recv_counts, rd.send_counts)
        recv_buf[0].index_copy_(0, recv_rows, recv)

    from osp_next_b200.parallel.p2p_collectives import p2p_redistribute
    rt_x = torch.randn(1, n, C, device=dev, requires_grad=True)
    g_out = torch.randn(1, lb.n_local, C, device=dev)
    y_keep = [None]

    def run_staged():
        with torch.no_grad():
            p2p_redistribute(rt_x, TOKEN, GROUP, grid, P, spec, ex)

    def run_staged_fwd_for_bwd():
        y_keep[0] = p2p_redistribute(rt_x, TOKEN, GROUP, grid, P, spec, ex)

    def run_staged_bwd():
        y_keep[0].backward(g_out, retain_graph=True)

    def run_nccl_xchg():
        send = out_local[0].index_select(0, send_rows)
        recv = torch.empty(int(sum(rd.recv_counts)), C, device=dev)
        dist.all_to_all_single(recv, send, rd.recv_counts, rd.send_counts)
        recv_buf[0].index_copy_(0, recv_rows, recv)

    res = {}
    run_staged_fwd_for_bwd()
    for name, fn in (("local", run_local), ("p2p", run_p2p), ("nccl", run_nccl), ("staged", run_staged),
                     ("staged_bwd", run_staged_bwd), ("nccl_xchg", run_nccl_xchg)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        ms = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ms.append(e0.elapsed_time(e1))
        t = torch.tensor([min(ms)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = float(t.item())
    err = ops.ext().get_error(local, True)
    flops = 2.0 * n * C * F
    remote_rows = int((rd.dest_rank != rank).sum().item())
    bytes_out = remote_rows * C * 4
    t_gemm = flops / (_peak_tflops() * 1e9)
    t_link = bytes_out / (NVLINK_GBS * 1e6)
    roof = max(t_gemm, t_link)
    hbm = (2 * n + lb.n_local) * C * 4                   # stage read + write, pull writes
    x_roof = max(t_link, hbm / (_hbm_gbs() * 1e6))
    if rank == 0:
        print(json.dumps({"bench": "ssp_exchange_training", "world": world, "rows_per_rank": n,
                          "ms_staged_fwd": round(res["staged"], 3), "ms_staged_bwd": round(res["staged_bwd"], 3),
                          "ms_nccl_exchange": round(res["nccl_xchg"], 3), "roofline_ms": round(x_roof, 3),
                          "frac_of_roofline_staged_fwd": round(x_roof / res["staged"], 3),
                          "frac_of_roofline_staged_bwd": round(x_roof / res["staged_bwd"], 3),
                          "frac_of_roofline_nccl": round(x_roof / res["nccl_xchg"], 3)}), flush=True)
        print(json.dumps({"bench": "ssp_exchange_ffn_down", "world": world, "rows_per_rank": n,
                          "remote_bytes_per_rank": bytes_out, "ms_local_gemm": round(res["local"], 3),
                          "ms_p2p_fused": round(res["p2p"], 3), "ms_nccl_path": round(res["nccl"], 3),
                          "roofline_ms": round(roof, 3), "roofline_terms_ms": [round(t_gemm, 3), round(t_link, 3)],
                          "frac_of_roofline_p2p": round(roof / res["p2p"], 3),
                          "frac_of_roofline_nccl": round(roof / res["nccl"], 3), "device_error": err}), flush=True)
    ex.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
