"""Op-level sweep of the fused row-parallel GEMM + all-reduce + residual +
RMSNorm prologue: M in {1, 8, 64, 512, 4096} rows, (K, N) in the Qwen2.5-14B
and -72B row-parallel shapes, over t tensor-parallel ranks.

    torchrun --nproc-per-node T -m tinybatch_b200.opbench [--rows 1,8,64,512,4096]

Y = X . W with X [M, K/t] and W [K/t, N] bf16 (values N(0,1)/sqrt(K), seed 2;
W is stored transposed, [N, K/t], the F.linear layout the kernels read),
summed over the t ranks, added to a residual and followed by the norm
prologue -- one kernel per rank.  Each row reports the device time per call
(CUDA graph of repeated calls, max over ranks), the same GEMM on one rank
without the exchange, the all-reduce bus bandwidth over the fused call
(`B_nvl / time`), and the fraction of the roofline

    T_roof = max(2 M (K/t) N / P_tensor,  B_hbm / BW_hbm,  B_nvl / BW_nvl)
    B_hbm  = 2 [(K/t) N + M (K/t) + 3 M N + N]      (bf16 bytes)
    B_nvl  = 2 (t-1)/t * 2 M N                       (all-reduce bus bytes)

with the measured HBM copy bandwidth and bf16 GEMM rate of MEASURED_PEAKS.json
and 770 GB/s per direction for NVLink (measured peer copy on this pool).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from . import ops
from .comm import TPComm
from .runtime import plan_gemm

NVLINK_GBS = 770.0
SHAPES = [(5120, 5120), (13824, 5120), (8192, 8192), (29568, 8192)]


def peaks() -> dict:
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    p = os.path.join(root, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def roofline_s(M: int, K: int, N: int, t: int, pk: dict) -> tuple[float, str]:
    kt = K // t
    flops = 2.0 * M * kt * N
    b_hbm = 2.0 * (kt * N + M * kt + 3 * M * N + N)
    b_nvl = 2.0 * (t - 1) / t * 2 * M * N
    terms = {"tensor": flops / (pk["bf16_tflops"] * 1e12), "hbm": b_hbm / (pk["hbm_gbs"] * 1e9),
             "nvlink": b_nvl / (NVLINK_GBS * 1e9) if t > 1 else 0.0}
    bound = max(terms, key=terms.get)
    return terms[bound], bound


def _time_graph(fn, reps: int, world: int) -> float:
    """Seconds per call of fn() (graph of `reps` calls, 3 replays, max over ranks)."""
    fn(0)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3 / (3 * reps)], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return float(t.item())


def run(ms: list[int], shapes=SHAPES, reps: int = 20, two_shot: bool | None = None) -> list[dict]:
    assert reps % 2 == 0, "an even number of calls per graph keeps the parities alternating"
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    dev = torch.device("cuda", torch.cuda.current_device())
    pk = peaks()
    out = []
    for K, N in shapes:
        comm = TPComm(rank, world, dev, N, max_rows=max(ms)) if world > 1 else None
        g = torch.Generator(device=dev).manual_seed(2)
        kt = K // world
        w = (torch.randn(N, kt, generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)
        gn = torch.ones(N, dtype=torch.bfloat16, device=dev)
        for M in ms:
            x = (torch.randn(M, kt, generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)
            h = torch.randn(M, N, generator=g, device=dev)
            hg = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            bn, splits = plan_gemm(M, N, kt)
            sq = torch.empty(ops.row_parts(N, bn, splits), M, device=dev)

            def plain(i):
                ops.row_linear_residual(x, w, h, gn, hg, sq, bn=bn, splits=splits)

            t_plain = _time_graph(plain, reps, world)
            t_fused = None
            if comm is not None:
                def fused(i):
                    # seq left to the communicator: consecutive calls alternate parity
                    # (graphs of an even number of calls keep that across replays)
                    comm.row_linear_residual(x, w, h, gn, hg, sq, bn=bn, splits=splits,
                                             two_shot=two_shot)
                t_fused = _time_graph(fused, reps, world)
            t = t_fused if t_fused is not None else t_plain
            t_roof, bound = roofline_s(M, K, N, world, pk)
            b_nvl = 2.0 * (world - 1) / world * 2 * M * N
            ts = (comm.use_two_shot(M, N) if two_shot is None else two_shot) if comm else None
            out.append({"M": M, "K": K, "N": N, "tp": world, "bn": bn, "splits": splits,
                        "two_shot": ts,
                        "us_fused": None if t_fused is None else round(t_fused * 1e6, 2),
                        "us_gemm_only": round(t_plain * 1e6, 2),
                        "us_roofline": round(t_roof * 1e6, 2), "bound": bound,
                        "frac": round(t_roof / t, 4),
                        # all-reduce bus bytes over the whole fused call (NCCL's busBw)
                        "nvl_bus_GBps": round(b_nvl / t / 1e9, 1) if world > 1 else None,
                        "peaks": pk["source"]})
        if comm is not None:
            comm.close()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", default="1,8,64,512,4096")
    ap.add_argument("--shapes", default="all", help="'all' or K,N (e.g. 5120,5120)")
    ap.add_argument("--two-shot", choices=["auto", "0", "1"], default="auto")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    shapes = SHAPES if args.shapes == "all" else [tuple(int(v) for v in args.shapes.split(","))]
    ts = None if args.two_shot == "auto" else args.two_shot == "1"
    rows = run([int(m) for m in args.rows.split(",")], shapes, two_shot=ts)
    if int(os.environ.get("RANK", "0")) == 0:
        for r in rows:
            print(json.dumps(r), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
