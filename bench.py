#!/usr/bin/env python
"""Benchmark of the GDN3 recurrent-scan hot path on B200.

Headline (BASELINE metric "chunked-scan prefill tok/s ... ; decode-step HBM GB/s"):
  * prefill: config 1 -- one GDN3 linear-attention layer scan, B=8, T=4096,
    H=16 heads x M=4 lanes, d_k=d_v=128, bf16 q/k/v/beta/log-decay (lane
    shared q/k/v), fp32 state, bf16 per-lane outputs, lane RoPE (first 64 dims
    on lane 0).  One step = one scan of the batch.  value = B*T tokens/s over
    all ranks (weak scaling: every rank scans its own config-1 shard).
  * decode (reported beside it): config 3 -- 24 layers x B=256 x H=16 x 4
    lanes, fp32 128x128 states, one token; GB/s of algorithmic traffic.

Timing: W warm-up steps, then exactly K steps between CUDA events on the
launching stream, barrier + synchronize on both sides, max over ranks.
Inputs (402 MB) and outputs (537 MB) exceed the 126 MB L2, so no flush is
needed between steps.  ``--impl reference`` times the CPU restatement of the
reference recurrence (the oracle port; the reference is pure Python/PyTorch)
on the host cores, on a bounded T-slice of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG1 = dict(B=8, T=4096, H=16, M=4, K=128, V=128, chunk=64)
CFG3 = dict(layers=24, B=256, H=16, M=4, K=128, V=128)


def chunk_flops_per_chain_token(dk, dv, C):
    """Algorithmic FLOPs of the chunked scan per chain-token (dense tiles, no C^3 solve)."""
    return 6 * dk * dv + 2 * C * (3 * dk + 2 * dv)


def wy_pieces(n_chains):
    """Launch pairs (pass 1 + pass 2) one prefill call makes: the library cuts the chains into
    single-wave pieces (one pass-2 CTA per SM) when at most 8 are needed."""
    forced = int(os.environ.get("GDNX_WY_PIECES", "0") or 0)
    if forced > 0:
        return min(forced, 8)
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    p = -(-n_chains // sms)
    return 1 if p > 8 else p


def kr_flops_per_chain_token(P, R=4, av=16, ak=16, bv=8, bk=8, K=128, V=128):
    """GDN3-KR algorithmic FLOPs per chain-token with chunk = compaction period P."""
    f_compact = 2 * R * (av * ak) * (bv * bk) + 2 * V * K * P + 2 * (1 + 2 * 2) * (av * ak) * (bv * bk) * (R + 4)
    return 4 * R * (av * ak * bk + av * bk * bv) + 4 * P * (K + V) + 2 * P * (2 * K + V) + f_compact / P


def prefill_bytes(c):
    """q,k,v read once per head (bf16), beta + log-decay per lane (bf16), bf16 per-lane outputs."""
    B, T, H, M, K, V = (c[x] for x in "BTHMKV")
    return B * T * H * ((2 * K + V) * 2 + M * 2 * 2 + M * V * 2)


def decode_bytes(c):
    L, B, H, M, K, V = (c[x] for x in ("layers", "B", "H", "M", "K", "V"))
    N = B * H * M
    return L * (2 * N * V * K * 4 + B * H * (2 * K + V) * 2 + N * 2 * 2 + N * V * 2)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm=d["hbm_gbs"], bf16=d["bf16_tflops"], bf16_sust=d.get("bf16_tflops_sustained"),
                    source="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sust=1400.0, source="fallback")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        time.sleep(0.25)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = [r for r in self.rows if len(r) >= 7]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][1]) if rows[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


CPU_SAMPLE = dict(B=1, T=512)  # one batch row of config 1 (all 64 chains), first 512 tokens


def cpu_sample_inputs():
    from oracle.inputs import scan_inputs, expand_lanes
    c = CFG1
    inp = scan_inputs(CPU_SAMPLE["B"], CPU_SAMPLE["T"], c["H"], c["M"], c["K"], c["V"], seed=1, dtype=torch.bfloat16)
    return expand_lanes(inp, c["M"])


def cpu_sample_rate(target_s):
    """Oracle port (CPU restatement of the reference's frozen loop, dense case) on the
    fixed config-1 slice CPU_SAMPLE, repeated for about ``target_s`` seconds; returns
    (tok/s, threads, sample description)."""
    from oracle import recurrence as R
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    ins = cpu_sample_inputs()
    R.dense_scan(*ins)
    reps, t0 = 0, time.perf_counter()
    while True:
        R.dense_scan(*ins)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= target_s:
            break
    tok = CPU_SAMPLE["B"] * CPU_SAMPLE["T"]
    return tok * reps / dt, threads, (f"config-1 slice B={CPU_SAMPLE['B']},T={CPU_SAMPLE['T']},H=16,M=4,d=128 "
                                     f"x{reps} ({dt:.1f} s)")


def run_reference(args, rank):
    """--impl reference: the reference recurrence restated on the CPU (rank 0 only)."""
    if rank != 0:
        return
    from oracle import recurrence as R
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    ins = cpu_sample_inputs()
    c = CFG1
    T = CPU_SAMPLE["T"]
    for _ in range(args.warmup):
        R.dense_scan(*ins)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        R.dense_scan(*ins)
    dt = (time.perf_counter() - t0) / args.steps
    sample = f"config-1 slice B={CPU_SAMPLE['B']},T={T},H=16,M=4,d=128 per step"
    value = CPU_SAMPLE["B"] * T / dt
    line = {"impl": "reference", "metric": "chunked-scan prefill tok/s", "value": value, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "config1-prefill slice", "B": CPU_SAMPLE["B"], "T": T,
                                            "H": c["H"], "M": c["M"], "K": c["K"], "V": c["V"]},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def make_prefill_inputs(c, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    B, T, H, M, K, V = (c[x] for x in "BTHMKV")
    bf = torch.bfloat16
    q = torch.nn.functional.normalize(torch.randn(B, T, H, K, device=dev, generator=g), dim=-1).to(bf)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, K, device=dev, generator=g), dim=-1).to(bf)
    v = torch.randn(B, T, H, V, device=dev, generator=g).to(bf)
    beta = torch.sigmoid(torch.randn(B, T, H, M, device=dev, generator=g)).to(bf)
    tau = torch.tensor([0.05, 0.02, 0.005, 0.001][:M], device=dev)
    logg = (-torch.nn.functional.softplus(torch.randn(B, T, H, M, device=dev, generator=g)) * tau).to(bf)
    return dict(q=q, k=k, v=v, beta=beta, logg=logg)


def timed(fn, steps, warmup, stream, barrier):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--algo", default="auto", choices=["auto", "recurrent", "chunked"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-kr", action="store_true")
    ap.add_argument("--kr-T", type=int, default=65536)
    ap.add_argument("--prefill-B", type=int, default=None, help="override B (profiling runs only)")
    ap.add_argument("--prefill-T", type=int, default=None, help="override T (profiling runs only)")
    ap.add_argument("--decode-layers", type=int, default=None, help="override layers (profiling runs only)")
    ap.add_argument("--no-config4", dest="config4", action="store_false", help="skip the config-4 sharded prefill leg")
    ap.add_argument("--config4-T", type=int, default=None, help="override config-4 T (smoke runs only)")
    ap.add_argument("--config4-slabs", type=int, default=8)
    ap.add_argument("--no-peer-gather", action="store_true", help="skip the fused routing + peer-store gather leg")
    ap.add_argument("--no-config4-ref-1gpu", dest="config4_ref_1gpu", action="store_false",
                    help="skip timing the full config-4 scan on rank 0 alone (N > 1)")
    ap.add_argument("--dropins-B", type=int, default=None, help="override the drop-in legs' B (profiling runs only)")
    ap.add_argument("--no-dropins", dest="dropins", action="store_false",
                    help="skip the drop-in legs (module input forms)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    from gdnx_b200 import ops
    from gdnx_b200.prologue import lane_rope
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    barrier = (lambda: dist.barrier()) if dist else (lambda: None)
    stream = torch.cuda.current_stream(dev)
    peaks = load_peaks()

    # ---------------- prefill (config 1 per rank) ----------------
    c = dict(CFG1)
    if args.prefill_B:
        c["B"] = args.prefill_B
    if args.prefill_T:
        c["T"] = args.prefill_T
    inp = make_prefill_inputs(c, dev, seed=1 + rank)
    rope = lane_rope(c["M"], c["K"], c["K"], 0.5)
    y = torch.empty(c["B"], c["T"], c["H"], c["M"], c["V"], dtype=torch.bfloat16, device=dev)
    ws = None  # the library's per-stream workspace (T_e, T_w, Mq tiles of the parallel pass)

    def step():
        ops.gdn3_scan(inp["q"], inp["k"], inp["v"], inp["beta"], inp["beta"], inp["logg"], decay_kind="log",
                      rope=rope, out=y, algo=args.algo, workspace=ws)

    with ClockSampler(local) as clk:
        ms = timed(step, args.steps, args.warmup, stream, barrier)
    clocks = clk.summary()
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    tokens = c["B"] * c["T"] * world
    value = tokens / (ms * 1e-3)
    chain_tokens = c["B"] * c["T"] * c["H"] * c["M"]
    flops = chain_tokens * chunk_flops_per_chain_token(c["K"], c["V"], c["chunk"])
    achieved = flops / (ms * 1e-3) / 1e12
    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists():
        traffic = json.loads(tp.read_text()).get("prefill_config1_bytes_per_launch")
    roofline = {"bound": "tensor", "scope": "whole prefill step: wy_prep_kernel + wy_scan_kernel",
                "achieved": achieved, "peak": peaks["bf16"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16"], "traffic": traffic,
                "peak_source": f"{peaks['source']} bf16 burst", "flops_per_launch": flops,
                "alg_bytes_per_launch": prefill_bytes(c),
                "hbm_frac": prefill_bytes(c) / (ms * 1e-3) / 1e9 / peaks["hbm"]}

    # ---------------- end to end: host buffers through the public API ----------------
    e2e = None
    if not args.no_e2e:
        # the public host-to-host entry point: per-batch-row slices whose copies in and out
        # overlap the neighbouring slices' scans (ops.gdn3_scan_host)
        host = {n: t.cpu().pin_memory() for n, t in inp.items()}
        yh = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        h2d = sum(t.numel() * t.element_size() for t in host.values())
        d2h = yh.numel() * yh.element_size()

        def e2e_step():
            ops.gdn3_scan_host(host["q"], host["k"], host["v"], host["beta"], host["beta"], host["logg"],
                               out=yh, device=dev, decay_kind="log", rope=rope, algo=args.algo)

        ms_e2e = timed(e2e_step, max(3, args.steps // 3), 3, stream, barrier)
        if dist:
            t = torch.tensor([ms_e2e], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_e2e = t.item()
        e2e = {"value": tokens / (ms_e2e * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e,
               "api": "ops.gdn3_scan_host (pinned host in/out, copies overlapped with the scans)"}
        del host, yh

    # ---------------- all-gather of per-head outputs (multi-GPU only) ----------------
    gather = None
    if dist:
        full = torch.empty((world * y.shape[0],) + tuple(y.shape[1:]), dtype=y.dtype, device=dev)
        ms_g = timed(lambda: dist.all_gather_into_tensor(full, y), 3, 1, stream, barrier)
        t = torch.tensor([ms_g], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gather = {"ms": t.item(), "bytes_per_rank_received": (world - 1) * y.numel() * y.element_size(),
                  "collective": "nccl all_gather_into_tensor"}
        del full

    # ---------------- config 4: sharded prefill, fused lane epilogue, pipelined all-gather ----------------
    cfg4 = None
    if args.config4:
        c4 = dict(B=64, T=8192, H=16, M=4, K=128, V=128, chunk=64)
        if args.config4_T:
            c4["T"] = args.config4_T
        from gdnx_b200.distributed import shard_for
        sh = shard_for(c4["B"], c4["H"], world, rank)
        lc = dict(c4)
        lc["B" if sh.axis == "batch" else "H"] = sh.stop - sh.start
        inp4 = make_prefill_inputs(lc, dev, seed=4 + rank)
        gr = torch.Generator(device=dev).manual_seed(40 + rank)
        router = torch.randn(lc["B"], lc["T"], lc["H"], lc["M"], device=dev, generator=gr).to(torch.bfloat16)
        norm = 1 + 0.1 * torch.randn(lc["V"], device=dev, generator=gr)
        rope4 = lane_rope(lc["M"], lc["K"], lc["K"], 0.5)
        yfull = torch.empty(lc["B"], lc["T"], lc["H"], lc["M"], lc["V"], dtype=torch.bfloat16, device=dev)

        def scan_only():  # one call per rank over the whole sequence
            ops.gdn3_scan(inp4["q"], inp4["k"], inp4["v"], inp4["beta"], inp4["beta"], inp4["logg"], decay_kind="log",
                          rope=rope4, out=yfull)

        ms4 = timed(scan_only, 3, 3, stream, barrier)
        del yfull
        slabs = args.config4_slabs
        Ts = lc["T"] // slabs
        ybuf = [torch.empty(lc["B"], Ts, lc["H"], lc["M"], lc["V"], dtype=torch.bfloat16, device=dev) for _ in range(2)]
        rbuf = [torch.empty(lc["B"], Ts, lc["H"], lc["V"], dtype=torch.bfloat16, device=dev) for _ in range(2)]
        gbuf = [torch.empty((world * lc["B"], Ts, lc["H"], lc["V"]), dtype=torch.bfloat16, device=dev)
                for _ in range(2)] if dist else None
        st = torch.zeros(lc["B"] * lc["H"] * lc["M"], lc["V"], lc["K"], dtype=torch.float32, device=dev)
        comm = torch.cuda.Stream(dev)
        ev_scan = [torch.cuda.Event() for _ in range(2)]
        ev_comm = [torch.cuda.Event() for _ in range(2)]

        def slab(i, state):
            sl = slice(i * Ts, (i + 1) * Ts)
            _, so = ops.gdn3_scan(inp4["q"][:, sl], inp4["k"][:, sl], inp4["v"][:, sl], inp4["beta"][:, sl],
                                  inp4["beta"][:, sl], inp4["logg"][:, sl], decay_kind="log",
                                  rope=lane_rope(lc["M"], lc["K"], lc["K"], 0.5, pos0=i * Ts), state=state,
                                  return_state=True, out=ybuf[i % 2])
            return so

        def scan_route_gather():
            # slab i's lane routing (HBM-bound) and all-gather run on a second stream while
            # slab i+1 scans (tensor/latency-bound)
            state = st
            for i in range(slabs):
                if i >= 2:
                    stream.wait_event(ev_comm[i % 2])  # ybuf / rbuf [i % 2] consumed
                state = slab(i, state)
                ev_scan[i % 2].record(stream)
                with torch.cuda.stream(comm):
                    comm.wait_event(ev_scan[i % 2])
                    sl = slice(i * Ts, (i + 1) * Ts)
                    ops.lane_route(ybuf[i % 2], router[:, sl], norm, out=rbuf[i % 2])
                    if dist:
                        dist.all_gather_into_tensor(gbuf[i % 2], rbuf[i % 2])
                    ev_comm[i % 2].record(comm)
            stream.wait_stream(comm)

        ms4e = timed(scan_route_gather, 3, 3, stream, barrier)
        # the same pipeline with the routing kernel storing its rows straight into every
        # rank's copy of the full routed output over NVLink (one fused kernel per slab, no
        # separate all-gather), one small all-reduce at the end as the completion barrier
        ms4p = None
        if dist and sh.axis == "batch" and not args.no_peer_gather:
            from gdnx_b200.distributed import PeerBuffer
            Bl, T4, H4, V4 = lc["B"], lc["T"], lc["H"], lc["V"]
            pbuf = PeerBuffer((world * Bl, T4, H4, V4), torch.bfloat16, dev)
            flag = torch.zeros(1, device=dev)
            dests = [pbuf.dest(rank * Bl * T4 * H4 * V4 + i * Ts * H4 * V4, (Bl - 1) * T4 * H4 * V4 + Ts * H4 * V4)
                     for i in range(slabs)]

            def scan_route_scatter():
                state = st
                for i in range(slabs):
                    if i >= 2:
                        stream.wait_event(ev_comm[i % 2])  # ybuf [i % 2] consumed
                    state = slab(i, state)
                    ev_scan[i % 2].record(stream)
                    with torch.cuda.stream(comm):
                        comm.wait_event(ev_scan[i % 2])
                        sl = slice(i * Ts, (i + 1) * Ts)
                        ops.lane_route_scatter(ybuf[i % 2], router[:, sl], dests[i], (T4 * H4 * V4, H4 * V4, V4),
                                               torch.bfloat16, norm)
                        ev_comm[i % 2].record(comm)
                with torch.cuda.stream(comm):
                    dist.all_reduce(flag)  # every rank's rows have landed everywhere
                stream.wait_stream(comm)

            ms4p = timed(scan_route_scatter, 3, 3, stream, barrier)
            pbuf.close()
        ms4g = None
        if dist:
            ms4g = timed(lambda: dist.all_gather_into_tensor(gbuf[0], rbuf[0]), 3, 1, stream, barrier) * slabs
        vals = torch.tensor([ms4, ms4e, ms4g or 0.0, ms4p or 0.0], device=dev)
        if dist:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        ms4, ms4e, ms4g, ms4p = vals.tolist()
        tok4 = c4["B"] * c4["T"]
        f4 = c4["B"] * c4["T"] * c4["H"] * c4["M"] * chunk_flops_per_chain_token(128, 128, 64)
        gathered = world * rbuf[0].numel() * rbuf[0].element_size() * slabs  # bytes of the full routed output
        cfg4 = {"workload": "config4: B=64,T=%d,H=16,M=4 sharded (batch x head) over %d rank(s)" % (c4["T"], world),
                "scan_ms": ms4, "scan_tok_per_s": tok4 / (ms4 * 1e-3), "scan_tflops": f4 / (ms4 * 1e-3) / 1e12,
                "scan_tc_frac_per_rank": f4 / world / (ms4 * 1e-3) / 1e12 / peaks["bf16"],
                "e2e_ms_pipelined": ms4e, "e2e_tok_per_s": tok4 / (ms4e * 1e-3), "slabs": slabs,
                "epilogue": "gdnx_epilogue lane routing + head norm per slab (routed [B,T,H,V] bf16)",
                "allgather_ms_serial": ms4g if dist else None,
                "allgather_bytes_total": gathered if dist else None,
                "nccl_busbw_gbs": (gathered * (world - 1) / world / (ms4g * 1e-3) / 1e9) if dist else None,
                "collective": "nccl all_gather_into_tensor of routed slabs on a comm stream" if dist else None,
                "e2e_ms_pipelined_peer": ms4p or None,
                "e2e_tok_per_s_peer": (tok4 / (ms4p * 1e-3)) if ms4p else None,
                "peer_gather": ("gdnx_epilogue_scatter: routing + stores into every rank's copy over NVLink "
                                "(CUDA IPC peer mappings), one all-reduce barrier per step") if ms4p else None}
        if dist and args.config4_ref_1gpu:
            # the same full config-4 scan on one GPU (rank 0), for the per-N speed-up
            t1 = torch.zeros(1, device=dev)
            if rank == 0:
                full = dict(c4)
                inpf = make_prefill_inputs(full, dev, seed=4)
                yf = torch.empty(full["B"], full["T"], full["H"], full["M"], full["V"], dtype=torch.bfloat16, device=dev)
                t1[0] = timed(lambda: ops.gdn3_scan(inpf["q"], inpf["k"], inpf["v"], inpf["beta"], inpf["beta"],
                                                    inpf["logg"], decay_kind="log", rope=rope4, out=yf),
                              3, 3, stream, lambda: None)
                del inpf, yf
            barrier()
            dist.all_reduce(t1, op=dist.ReduceOp.MAX)
            cfg4["scan_ms_1gpu"] = t1.item()
            cfg4["scan_speedup_vs_1gpu"] = t1.item() / ms4
            cfg4["scan_efficiency"] = t1.item() / ms4 / world
        del inp4, ybuf, rbuf, gbuf, st, router

    # ---------------- decode (config 3) ----------------
    decode = None
    if not args.no_decode:
        d = dict(CFG3)
        if args.decode_layers:
            d["layers"] = args.decode_layers
        N = d["B"] * d["H"] * d["M"]
        g = torch.Generator(device=dev).manual_seed(3 + rank)
        states = [torch.randn(N, d["V"], d["K"], device=dev, generator=g) * 0.02 for _ in range(d["layers"])]
        bf = torch.bfloat16
        toks = []
        for _ in range(d["layers"]):
            qd = torch.nn.functional.normalize(torch.randn(d["B"], d["H"], d["K"], device=dev, generator=g), dim=-1).to(bf)
            kd = torch.nn.functional.normalize(torch.randn(d["B"], d["H"], d["K"], device=dev, generator=g), dim=-1).to(bf)
            vd = torch.randn(d["B"], d["H"], d["V"], device=dev, generator=g).to(bf)
            bd = torch.sigmoid(torch.randn(d["B"], d["H"], d["M"], device=dev, generator=g)).to(bf)
            tau = torch.tensor([0.05, 0.02, 0.005, 0.001], device=dev)
            ld = (-torch.nn.functional.softplus(torch.randn(d["B"], d["H"], d["M"], device=dev, generator=g)) * tau).to(bf)
            toks.append((qd, kd, vd, bd, ld))
        yd = [torch.empty(d["B"], d["H"], d["M"], d["V"], dtype=bf, device=dev) for _ in range(d["layers"])]
        drope = lane_rope(d["M"], d["K"], d["K"], 0.5, pos0=4096)

        def dstep():
            for l in range(d["layers"]):
                qd, kd, vd, bd, ld = toks[l]
                ops.decode_step(states[l], qd, kd, vd, bd, bd, ld, decay_kind="log", rope=drope, out=yd[l])

        dms = timed(dstep, max(3, args.steps // 3), 3, stream, barrier)
        if dist:
            t = torch.tensor([dms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dms = t.item()
        db = decode_bytes(d) * world
        decode = {"metric": "decode-step HBM GB/s", "value": db / (dms * 1e-3) / 1e9, "unit": "GB/s",
                  "ms_per_step": dms, "alg_bytes_per_step": db, "layers": d["layers"],
                  "states_per_layer": N, "hbm_frac": db / world / (dms * 1e-3) / 1e9 / peaks["hbm"],
                  "peak_gbs": peaks["hbm"], "launches_per_step": d["layers"]}
        del states

    # ---------------- Kronecker-residual scan (config 2, per rank) ----------------
    kr = None
    if not args.no_kr:
        kc = dict(B=1, T=args.kr_T, H=16, M=4, K=128, V=128)
        kin = make_prefill_inputs(kc, dev, seed=2 + rank)
        N = kc["B"] * kc["H"] * kc["M"]
        from gdnx_b200.gdn3_upgrade import reference_sketch
        krs = {}
        for P in (256, 16):
            G = reference_sketch(N, 64, 8, dev)
            st = ops.KRState.zeros(N, 4, P, (16, 16, 8, 8), 128, 128, dev)
            yk = torch.empty(kc["B"], kc["T"], kc["H"], kc["M"], kc["V"], dtype=torch.bfloat16, device=dev)

            def kstep():
                st.slot.zero_()
                ops.gdn3_kr_scan(kin["q"], kin["k"], kin["v"], kin["beta"], kin["beta"], kin["logg"], st, G, P=P,
                                 decay_kind="log", rope=rope)

            kms = timed(kstep, 2, 3, stream, barrier)
            kf = kc["B"] * kc["T"] * kc["H"] * kc["M"] * kr_flops_per_chain_token(P)
            krs[f"P{P}"] = {"ms_per_call": kms, "tok_per_s": kc["B"] * kc["T"] * world / (kms * 1e-3),
                            "tflops_by_formula": kf / (kms * 1e-3) / 1e12,
                            "tc_frac": kf / (kms * 1e-3) / 1e12 / peaks["bf16"]}
        del kin
        # the GDN3 drop-in on what GDN3LinearAttn.forward passes: fp32 per-lane q/k/v, vector gates
        import types
        from gdnx_b200.gdn3_upgrade import gdn3_recurrent_state
        g2 = torch.Generator(device=dev).manual_seed(20 + rank)
        shp = (kc["B"], kc["T"], kc["H"], kc["M"], kc["K"])
        qx = torch.nn.functional.normalize(torch.randn(*shp, device=dev, generator=g2), dim=-1)
        kx = torch.nn.functional.normalize(torch.randn(*shp, device=dev, generator=g2), dim=-1)
        vx = torch.randn(*shp, device=dev, generator=g2)
        bg = torch.sigmoid(torch.randn(*shp, device=dev, generator=g2))
        wg = torch.sigmoid(torch.randn(*shp, device=dev, generator=g2))
        dec = 0.78 + 0.219 * torch.rand(*shp[:4], device=dev, generator=g2)
        layer = types.SimpleNamespace(R=4, P=256, a_v=16, a_k=16, b_v=8, b_k=8, slow_decay=0.97, compact_mode="svd")
        dms = timed(lambda: gdn3_recurrent_state(layer, qx, kx, vx, bg, wg, dec), 2, 3, stream, barrier)
        krs["dropin_P256_fp32_vector_gates"] = {
            "call": "gdn3_upgrade.gdn3_recurrent_state (T >= P: KR kernel)", "ms_per_call": dms,
            "tok_per_s": kc["B"] * kc["T"] * world / (dms * 1e-3)}
        del qx, kx, vx, bg, wg, dec
        kr = {"metric": "KR prefill tok/s (config 2)", "B": 1, "T": kc["T"], "H": 16, "M": 4,
              "state": "A 16x16 (x) B 8x8, R=4, + U,V 128xP, delta=0.97", **krs}

    # ---------------- the drop-ins on the input forms the reference modules pass ----------------
    dropins = None
    if args.dropins:
        from gdnx_b200 import kmd2_fast_scan
        from gdnx_b200.gdn3_upgrade import gdn3_recurrent_state
        import types
        B, T, H, dk = args.dropins_B or CFG1["B"], CFG1["T"], CFG1["H"], CFG1["K"]
        g = torch.Generator(device=dev).manual_seed(11 + rank)
        dropins = {}
        # KMD2NativeAttn.forward -> kmd2_fast_scan: fp32 q [B,T,H,4,dk] (scaled), k, v, per-channel g
        q = torch.nn.functional.normalize(torch.randn(B, T, H, 4, dk, device=dev, generator=g), dim=-1) * dk ** -0.5
        k = torch.nn.functional.normalize(torch.randn(B, T, H, dk, device=dev, generator=g), dim=-1)
        v = torch.randn(B, T, H, dk, device=dev, generator=g)
        gd = torch.exp(-torch.nn.functional.softplus(1.2 * torch.randn(B, T, H, dk, device=dev, generator=g) - 0.6))
        be = torch.sigmoid(torch.randn(B, T, H, device=dev, generator=g))
        bw = torch.sigmoid(torch.randn(B, T, H, device=dev, generator=g))
        mix = torch.randn(H, 4, device=dev, generator=g)
        kms = timed(lambda: kmd2_fast_scan.scan_with_update_norm(q, k, v, gd, be, bw, mix), 5, 3, stream, barrier)
        kf = B * T * H * chunk_flops_per_chain_token(dk, dk, 64)
        dropins["kmd2_fast_scan"] = {
            "call": "kmd2_fast_scan.scan_with_update_norm", "shape": f"B={B},T={T},H={H},r_out=4,dk=dv={dk} fp32, "
            "per-channel decay, scores", "kernels": "wyg_prep_kernel + wyg_chain_kernel", "ms": kms,
            "tok_per_s": B * T / (kms * 1e-3), "tflops": kf / (kms * 1e-3) / 1e12}
        # training step of the same call: forward + exact fp32 backward (gdnx_scan_bwd)
        for t_ in (q, k, v, gd, be, bw, mix):
            t_.requires_grad_(True)
        gyk = torch.randn(B, T, H, dk, device=dev, generator=g)

        def kmd2_train():
            yk = kmd2_fast_scan.scan(q, k, v, gd, be, bw, mix)
            yk.backward(gyk)

        tms = timed(kmd2_train, 2, 1, stream, barrier)
        dropins["kmd2_fast_scan_fwd_bwd"] = {
            "call": "kmd2_fast_scan.scan + backward (autograd)", "shape": dropins["kmd2_fast_scan"]["shape"],
            "kernels": "wyg_prep_kernel + wyg_chain_kernel + scan_bwd_kernel", "ms": tms,
            "tok_per_s": B * T / (tms * 1e-3)}
        del q, k, v, gd, be, bw, gyk
        # GDN3LinearAttn with bf16 features: per-lane rotated q/k, vector erase/write gates
        M = CFG1["M"]
        bf = torch.bfloat16
        qx = torch.nn.functional.normalize(torch.randn(B, T, H, M, dk, device=dev, generator=g), dim=-1).to(bf)
        kx = torch.nn.functional.normalize(torch.randn(B, T, H, M, dk, device=dev, generator=g), dim=-1).to(bf)
        vx = torch.randn(B, T, H, M, dk, device=dev, generator=g).to(bf)
        bg = torch.sigmoid(torch.randn(B, T, H, M, dk, device=dev, generator=g)).to(bf)
        wg = torch.sigmoid(torch.randn(B, T, H, M, dk, device=dev, generator=g)).to(bf)
        dec = 0.78 + 0.219 * torch.rand(B, T, H, M, device=dev, generator=g)
        layer = types.SimpleNamespace(R=4, P=1 << 30, a_v=16, a_k=16, b_v=8, b_k=8, slow_decay=0.97,
                                      compact_mode="svd")
        gms = timed(lambda: gdn3_recurrent_state(layer, qx, kx, vx, bg, wg, dec), 5, 3, stream, barrier)
        gf = B * T * H * M * chunk_flops_per_chain_token(dk, dk, 64)
        dropins["gdn3_bf16_vector_gates"] = {
            "call": "gdn3_upgrade.gdn3_recurrent_state (T < P: dense)", "shape": f"B={B},T={T},H={H},M={M},d={dk} "
            "bf16 per-lane q/k/v, vector b/w gates, gamma decay", "kernels": "wyg_prep_kernel + wyg_chain_kernel",
            "ms": gms, "tok_per_s": B * T / (gms * 1e-3), "tflops": gf / (gms * 1e-3) / 1e12}
        qx, kx, vx, bg, wg = (t.float() for t in (qx, kx, vx, bg, wg))
        fms = timed(lambda: gdn3_recurrent_state(layer, qx, kx, vx, bg, wg, dec), 2, 1, stream, barrier)
        dropins["gdn3_fp32_exact"] = {
            "call": "gdn3_upgrade.gdn3_recurrent_state (T < P: dense)", "shape": "as above, fp32 features "
            "(what GDN3LinearAttn.forward passes)", "kernels": "recurrent_scan_kernel (exact fp32 contract)",
            "ms": fms, "tok_per_s": B * T / (fms * 1e-3)}
        del qx, kx, vx, bg, wg, dec

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, threads, sample = cpu_sample_rate(target_s=10.0)
        cpu = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": "chunked-scan prefill tok/s", "value": value, "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "config1: GDN3 dense prefill layer scan per rank", **c,
                           "rope": "lane RoPE, lane 0 first 64 dims base 10000",
                           "state": "fp32", "io": "bf16", "algo": args.algo,
                           "l2": "inputs 402 MB + outputs 537 MB > 126 MB L2 (no flush)",
                           "parallelism": f"(batch x head) shards, dp{world}"},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": 2 * wy_pieces(c["B"] * c["H"] * c["M"]) * args.steps,
                "clocks": clocks, "decode": decode, "gather": gather, "kr": kr, "config4": cfg4, "dropins": dropins}
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
