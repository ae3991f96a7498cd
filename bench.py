#!/usr/bin/env python
"""Decode state-op benchmark of the tiered Mamba2 state update (nested_ssm "v4").

Metric: decode state-op tokens/s at B=448 over 27 Mamba2 layers,
Nemotron-Nano-9B-v2 shapes (H=128, P=80, N=128, G=8), hot 32 dims fp32, cold 96
dims fp8 e4m3 with one fp32 scale per (seq, head, headdim row), c=4.  One step =
one decode token through all 27 layers' state ops (rotation of B and C by R, the
tiered update with its ring write and rank-c flush).  Synthetic seeded inputs with
the BASELINE distributions; the state pool (29 GB) is far larger than L2, so no
L2 flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun: every rank owns its own slot pool and batch of 448
(weak scaling, no data-path collective).

Besides the headline step the line carries: `e2e` (the same step through the public API
with host copies), `cpu_baseline` (the oracle port on the host cores), `fresh_control`
(the untiered fp32 update), `conv_step`, `prefill_scan` (the chunked prefill scan) and
`ragged` (a continuous-batching run over a slot pool with finishes, admissions and per-slot
flush phases); `--no-<leg>` skips one.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402

H, P, N, G = 128, 80, 128, 8
METRIC = "decode state-op tokens/s at B=448 (27 layers)"
# Published reference number for this exact configuration: tiered fp8-cold c=4 at
# B=448 ran at 0.68x the fla fresh op of 51.45 ms/step (8,707 tok/s): 5,921 tok/s.
REF_PUBLISHED_TOKS = 0.68 * 8707.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=448)
    ap.add_argument("--layers", type=int, default=27)
    ap.add_argument("--chunk", type=int, default=4)
    ap.add_argument("--hot", type=int, default=32)
    ap.add_argument("--cold", choices=["fp8", "bf16", "fp32"], default="fp8")
    ap.add_argument("--no-fresh", action="store_true", help="skip the untiered fresh control")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-conv", action="store_true", help="skip the decode-token conv measurement")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--cpu-sample-batch", type=int, default=4)
    ap.add_argument("--cpu-leg-only", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of replaying CUDA graphs")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill chunked-scan measurement")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the prefill chunked-scan leg and print its JSON (profiling)")
    ap.add_argument("--prefill-batch", type=int, default=64)
    ap.add_argument("--prefill-len", type=int, default=2048)
    ap.add_argument("--prefill-reps", type=int, default=0, help="timed launches (0: from --steps)")
    ap.add_argument("--no-ragged", action="store_true", help="skip the continuous-batching ragged leg")
    ap.add_argument("--ragged-slots", type=int, default=2048, help="slot pool per GPU of the ragged leg")
    ap.add_argument("--ragged-steps", type=int, default=512, help="timed steps of the ragged leg")
    ap.add_argument("--no-config1", action="store_true", help="skip the B=256 / 256-step configuration")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip the same-box run of the reference's own GPU decode arms")
    ap.add_argument("--reference-gpu-leg-only", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--no-multi-gpu-check", action="store_true")
    ap.add_argument("--no-selfspec", action="store_true")
    ap.add_argument("--model-e2e", action="store_true",
                    help="only the end-to-end model decode (reduced BASELINE config 4) and print its JSON")
    ap.add_argument("--model-batch", type=int, default=448)
    ap.add_argument("--model-prompt", type=int, default=8)
    ap.add_argument("--model-gen", type=int, default=32)
    ap.add_argument("--model-arms", default="ours,reference,hf")
    ap.add_argument("--vllm-e2e", action="store_true",
                    help="only the serving-engine decode (vLLM 0.22, stock against the tiered hook) and print its JSON")
    ap.add_argument("--vllm-arms", default="vllm,ours")
    ap.add_argument("--vllm-mem", type=float, default=0.6, help="vLLM gpu_memory_utilization, stock arm")
    ap.add_argument("--vllm-mem-ours", type=float, default=0.72,
                    help="vLLM gpu_memory_utilization with the hook (its tiered pools, max_num_seqs + 64 slots "
                         "per layer, are allocated after vLLM's cache)")
    ap.add_argument("--vllm-blocks", type=int, default=0, help="vLLM num_gpu_blocks_override (0: vLLM's choice)")
    ap.add_argument("--vllm-arm", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--vllm-model", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--vllm-tokens", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--vllm-eager", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--vllm-reinit", action="store_true",
                    help="replace vLLM's dummy weights by seeded BASELINE-distribution weights (token checks)")
    return ap.parse_args()


# --------------------------------------------------------------------------
# algorithmic bytes (per token, per layer, per sequence) of the tiered step kernel
# --------------------------------------------------------------------------
def step_bytes_per_seq(c: int, pb: int, cold: str, io_bytes: int = 2, out_bytes: int = 2) -> float:
    """Algorithmic HBM bytes of one tiered state update (STEP + FLUSH launches) for one
    sequence-token-layer, averaged over a c-token cycle.

    STEP: hot read+write, cold (+ row scales) read, x / dt / rotated B, C in, y out,
    glog and t read+write, this token's ring entry written.  FLUSH (once per c tokens):
    cold (+ scales) read and written, the c ring entries read."""
    s = {"fp8": 1, "bf16": 2, "fp32": 4}[cold]
    Nc = N - pb
    scale = H * P * 4 if cold == "fp8" else 0
    ring_w = H * P * io_bytes + H * 4 + G * Nc * io_bytes
    step = (2 * H * P * pb * 4 + H * P * Nc * s + scale + H * P * io_bytes + H * 2
            + 2 * G * N * io_bytes + H * P * out_bytes + 2 * H * 4 + 2 * H * 4 + ring_w)
    flush = 2 * (H * P * Nc * s + scale) + c * ring_w
    return step + flush / c


def reference_model_bytes_per_seq(c: int) -> float:
    """Byte model the reference's design implies (separate flush, fp32 ring)."""
    return 3_780_872 + 2_048_000 / c


def fresh_bytes_per_seq(io_bytes=2, out_bytes=2) -> float:
    return 2 * H * P * N * 4 + H * P * io_bytes + H * 2 + 2 * G * N * io_bytes + H * P * out_bytes


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_tensor_peak() -> float:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    return 1590.0


def load_traffic():
    """Per-launch DRAM bytes of the step kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return None


# --------------------------------------------------------------------------
# clocks sampled during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        # nvidia-smi numbers GPUs physically; address ours by UUID
        self.idx = str(gpu_index)
        try:
            u = str(torch.cuda.get_device_properties(gpu_index).uuid)
            self.idx = u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            pass
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", self.idx], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for nm, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()) if rows else None,
                "reasons": sorted(reasons)}


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------
def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, ws, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, ws: int) -> float:
    if ws == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------
# workload
# --------------------------------------------------------------------------
class Workload:
    """L layers of state ops for B sequences on this rank, inputs resident in HBM."""

    NI = 4  # distinct per-step input sets cycled through

    def __init__(self, args, rank: int):
        from nested_ssm_b200 import TieredSlotPool, prefill_split
        self.args = args
        dev = torch.device("cuda")
        L, B = args.layers, args.batch
        self.L, self.B = L, B
        gen = torch.Generator(device=dev)
        gen.manual_seed(1000 + rank)
        self.pool = TieredSlotPool(L, B, H, P, N, G, args.hot, args.chunk, args.cold, torch.bfloat16, dev,
                                   max_batch=B)
        slots = torch.arange(B, dtype=torch.int32, device=dev)
        self.slots = slots
        # per-layer parameters with the BASELINE distributions
        self.A, self.D, self.dtb, self.R = [], [], [], []
        for l in range(L):
            self.A.append(-torch.exp(torch.rand(H, device=dev, generator=gen) * math.log(16.0)))
            self.D.append(torch.randn(H, device=dev, generator=gen))
            u = torch.rand(H, device=dev, generator=gen) * (0.1 - 1e-3) + 1e-3
            self.dtb.append(torch.log(torch.expm1(u)))
            self.R.append(torch.linalg.qr(torch.randn(G, N, N, device=dev, generator=gen))[0].contiguous())
            # prefill: initial state ~ N(0, 0.1), split into hot fp32 / cold fp8
            st = torch.randn(B, H, P, N, device=dev, generator=gen) * math.sqrt(0.1)
            prefill_split(self.pool, l, st, slots)
            del st
        NI = self.NI
        self.x = torch.randn(NI, L, B, H, P, device=dev, generator=gen).to(torch.bfloat16)
        self.dt = torch.randn(NI, L, B, H, device=dev, generator=gen).to(torch.bfloat16)
        self.BC = (torch.randn(NI, L, 2 * B, G * N, device=dev, generator=gen) / math.sqrt(N)).to(torch.bfloat16)
        self.BCr = torch.empty(2 * B, G * N, dtype=torch.bfloat16, device=dev)
        self.y = torch.empty(L, B, H, P, dtype=torch.bfloat16, device=dev)
        torch.cuda.synchronize()

    def layer(self, l: int, k: int, ev=None):
        """One layer's state op for input set k: rotation (one launch for B and C) then
        the tiered step kernel."""
        from nested_ssm_b200 import rot_flat, tiered_state_update
        i = k % self.NI
        B = self.B
        if ev is not None:
            ev[0].record()
        rot_flat(self.BC[i, l], self.R[l], out=self.BCr)
        if ev is not None:
            ev[1].record()
        tiered_state_update(self.pool, l, self.x[i, l], self.dt[i, l], self.A[l], self.BCr[:B].view(B, G, N),
                            self.BCr[B:].view(B, G, N), self.D[l], self.dtb[l], True, self.slots, -1, self.y[l],
                            None, 1e-3)
        if ev is not None:
            ev[2].record()

    def step(self, k: int, evs=None):
        for l in range(self.L):
            self.layer(l, k, None if evs is None else evs[l])


def time_fresh(args, rank: int, ws: int):
    """Untiered fp32 fresh update (own kernel) on the same shapes: tokens/s."""
    from nested_ssm_b200 import rot_flat, selective_state_update
    dev = torch.device("cuda")
    L, B = args.layers, args.batch
    gen = torch.Generator(device=dev)
    gen.manual_seed(2000 + rank)
    state = torch.empty(L, B, H, P, N, device=dev)
    for l in range(L):
        state[l].normal_(0.0, math.sqrt(0.1), generator=gen)
    A = -torch.exp(torch.rand(L, H, device=dev, generator=gen) * math.log(16.0))
    D = torch.randn(L, H, device=dev, generator=gen)
    dtb = torch.log(torch.expm1(torch.rand(L, H, device=dev, generator=gen) * (0.1 - 1e-3) + 1e-3))
    R = [torch.linalg.qr(torch.randn(G, N, N, device=dev, generator=gen))[0].contiguous() for _ in range(L)]
    x = torch.randn(L, B, H, P, device=dev, generator=gen).to(torch.bfloat16)
    dt = torch.randn(L, B, H, device=dev, generator=gen).to(torch.bfloat16)
    BC = (torch.randn(L, 2 * B, G * N, device=dev, generator=gen) / math.sqrt(N)).to(torch.bfloat16)
    BCr = torch.empty(2 * B, G * N, dtype=torch.bfloat16, device=dev)
    y = torch.empty(L, B, H, P, dtype=torch.bfloat16, device=dev)
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(L)]
    kdur = []

    def step(timed=False):
        for l in range(L):
            if timed:
                evs[l][0].record()
            rot_flat(BC[l], R[l], out=BCr)
            if timed:
                evs[l][1].record()
            selective_state_update(state[l], x[l], dt[l], A[l], BCr[:B].view(B, G, N), BCr[B:].view(B, G, N),
                                   D[l], None, dtb[l], True, slots, -1, y[l])
            if timed:
                evs[l][2].record()

    K = max(4, args.steps // 4)
    for _ in range(max(3, args.warmup // 2)):
        step()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        step(timed=True)
        torch.cuda.synchronize()
        kdur += [evs[l][1].elapsed_time(evs[l][2]) for l in range(L)]
    e1.record()
    torch.cuda.synchronize()
    # the per-step syncs above add host gaps: time once more without them
    e0.record()
    for _ in range(K):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / K, ws)
    barrier(ws)
    del state, x, BC, y
    torch.cuda.empty_cache()
    kms = statistics.mean(kdur)
    return {"tokens_per_s": ws * B / (ms / 1e3), "ms_per_step": ms,
            "kernel_ms": kms, "kernel_gbs": B * fresh_bytes_per_seq() / (kms / 1e3) / 1e9}


def conv_bytes_per_row(L: int = 3) -> int:
    """Algorithmic HBM bytes of the decode-token conv per sequence-layer (bf16): the conv
    state read and written, the in_proj slice read, x / B' / C' written."""
    D = H * P + 2 * G * N
    return 2 * D * L * 2 + D * 2 + D * 2


def time_conv(args, rank: int, ws: int):
    """nssm_conv_step (conv1d update + SiLU + split + rotation, one launch) at the bench's
    batch over all layers' conv states (891 MB at B=448: larger than L2)."""
    from nested_ssm_b200 import conv_step
    dev = torch.device("cuda")
    L, B, K, Ls = args.layers, args.batch, 4, 3
    D = H * P + 2 * G * N
    gen = torch.Generator(device=dev)
    gen.manual_seed(3000 + rank)
    state = (torch.randn(L, B, D, Ls, device=dev, generator=gen) * 0.5).to(torch.bfloat16)
    w = (torch.rand(L, D, K, device=dev, generator=gen) - 0.5).to(torch.bfloat16)
    bias = (torch.randn(L, D, device=dev, generator=gen) * 0.1).to(torch.bfloat16)
    R = [torch.linalg.qr(torch.randn(G, N, N, device=dev, generator=gen))[0].contiguous() for _ in range(L)]
    xbc = torch.randn(L, B, D, device=dev, generator=gen).to(torch.bfloat16)
    x = torch.empty(B, H, P, dtype=torch.bfloat16, device=dev)
    Bo = torch.empty(B, G, N, dtype=torch.bfloat16, device=dev)
    Co = torch.empty_like(Bo)
    slots = torch.arange(B, dtype=torch.int32, device=dev)

    def run():
        for l in range(L):
            conv_step(xbc[l], state[l], w[l], bias[l], "silu", slots, -1, R[l], nheads=H, headdim=P,
                      ngroups=G, dstate=N, x_out=x, B_out=Bo, C_out=Co)

    for _ in range(3):
        run()
    barrier(ws)
    torch.cuda.synchronize()
    reps = max(4, args.steps // 4)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / (reps * L), ws)
    barrier(ws)
    del state, w, xbc
    torch.cuda.empty_cache()
    peak, kind = load_peaks()
    gbs = B * conv_bytes_per_row(Ls) / (ms / 1e3) / 1e9
    return {"ms_per_launch": round(ms, 4), "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
            "bytes_per_launch": B * conv_bytes_per_row(Ls), "width": K, "state_len": Ls,
            "kernel": "conv_step_kernel (conv1d update + SiLU + split + rotation of B and C)"}


def prefill_bytes_per_token(io_bytes=2, dt_bytes=2) -> int:
    """Algorithmic HBM bytes of the chunked scan per token-layer: x, B, C, dt in, y out (the
    final state, H*P*N*4 per sequence, is added per launch)."""
    return H * P * io_bytes + 2 * G * N * io_bytes + H * dt_bytes + H * P * io_bytes


def prefill_flops_per_chunk(Q=128) -> int:
    """Tensor-core FLOPs of one 128-token chunk of one sequence (mamba_ssm's algorithm:
    C.B^T once per group; C.S_prev, M.x and the chunk state B_s^T.x per head)."""
    return G * 2 * Q * Q * N + H * 3 * 2 * Q * N * P


def time_prefill(args, rank: int, ws: int):
    """nssm_chunk_scan (one layer's prefill scan, tcgen05) on a [batch, len] prompt batch: x, B,
    C as views of one conv output and dt of one in_proj slice (the reference's layout), y and
    the fp32 final states written; inputs and outputs larger than L2."""
    from nested_ssm_b200 import mamba_chunk_scan_combined
    dev = torch.device("cuda")
    Bp, T = args.prefill_batch, args.prefill_len
    I, GN = H * P, G * N
    gen = torch.Generator(device=dev)
    gen.manual_seed(4000 + rank)
    xbc = torch.empty(Bp, T, I + 2 * GN, dtype=torch.bfloat16, device=dev)
    xbc[..., :I].normal_(generator=gen)
    xbc[..., I:].normal_(std=N ** -0.25, generator=gen)
    dt = torch.randn(Bp, T, H, device=dev, generator=gen).to(torch.bfloat16)
    A = -torch.exp(torch.rand(H, device=dev, generator=gen) * math.log(16.0))
    D = torch.randn(H, device=dev, generator=gen)
    dt_bias = torch.log(torch.expm1(torch.rand(H, device=dev, generator=gen) * (0.1 - 1e-3) + 1e-3))
    x = xbc[..., :I].view(Bp, T, H, P)
    Bv = xbc[..., I:I + GN].view(Bp, T, G, N)
    Cv = xbc[..., I + GN:].view(Bp, T, G, N)
    y = torch.empty(Bp, T, H, P, dtype=torch.bfloat16, device=dev)
    fin = torch.empty(Bp, H, P, N, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def run():
        mamba_chunk_scan_combined(x, dt, A, Bv, Cv, 128, D=D, dt_bias=dt_bias, dt_softplus=True, out=y,
                                  final_states=fin, status=status)

    for _ in range(3):
        run()
    barrier(ws)
    torch.cuda.synchronize()
    reps = args.prefill_reps or max(3, args.steps // 8)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError(f"chunk scan reported status {int(status.item())}")
    ms = max_over_ranks(e0.elapsed_time(e1) / reps, ws)
    barrier(ws)
    del xbc, y, fin
    torch.cuda.empty_cache()
    peak, kind = load_peaks()
    tflops_peak = load_tensor_peak()
    nbytes = Bp * T * prefill_bytes_per_token() + Bp * H * P * N * 4
    flops = Bp * ((T + 127) // 128) * prefill_flops_per_chunk()
    gbs = nbytes / (ms / 1e3) / 1e9
    tfs = flops / (ms / 1e3) / 1e12
    traffic = None
    tr = (load_traffic() or {}).get("prefill_scan")
    if tr:   # captured on a smaller case: scale by the bytes the two launches move
        cap_bytes = tr["tokens"] * prefill_bytes_per_token() + tr["sequences"] * H * P * N * 4
        traffic = int(tr["bytes_per_launch"] * nbytes / cap_bytes)
    # whole-job throughput: every rank scans its own prompt batch (max-over-ranks time)
    return {"ms_per_launch": round(ms, 4), "tokens_per_s_per_layer": round(ws * Bp * T / (ms / 1e3), 1),
            "tokens_per_s_27_layers": round(ws * Bp * T / (27 * ms / 1e3), 1), "n_gpus": ws,
            "config": {"batch_per_gpu": Bp, "seqlen": T, "chunk_size": 128, "H": H, "P": P, "N": N, "G": G,
                       "dtype": "bf16 x/B/C/y, fp32 accumulate and state", "layout": "x/B/C views of conv output"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_kind": kind, "bytes_per_launch": nbytes,
                         "traffic": traffic,
                         "tensor_tflops": round(tfs, 1), "tensor_frac": round(tfs / tflops_peak, 4),
                         "flops_per_launch": flops},
            "gpu_launches_per_layer": 1,
            "kernel": "chunk_scan_kernel (tcgen05: C.B^T, C.S_prev, M.x, B_s^T.x per 128-token chunk)"}


def gpu_local_cpus(device_index: int) -> list[int] | None:
    """Host CPUs on the GPU's NUMA node (sysfs ``local_cpulist`` of its PCI device), or None
    when the platform does not say."""
    try:
        pr = torch.cuda.get_device_properties(device_index)
        path = "/sys/bus/pci/devices/%04x:%02x:%02x.0/local_cpulist" % (pr.pci_domain_id, pr.pci_bus_id,
                                                                      pr.pci_device_id)
        with open(path) as f:
            txt = f.read().strip()
    except (OSError, AttributeError, RuntimeError):
        return None
    cpus = []
    for part in txt.split(","):
        if "-" in part:
            a, b = part.split("-")
            cpus.extend(range(int(a), int(b) + 1))
        elif part:
            cpus.append(int(part))
    allowed = os.sched_getaffinity(0)
    cpus = [c for c in cpus if c in allowed]
    return cpus or None


def pinned_near_gpu(tensors, device_index: int):
    """Pinned host copies of ``tensors`` whose pages are first touched by a thread running on
    the GPU's own NUMA node (the kernel places pages where they are first written)."""
    cpus = gpu_local_cpus(device_index)
    old = os.sched_getaffinity(0)
    try:
        if cpus:
            os.sched_setaffinity(0, cpus)
        return [t.cpu().pin_memory() if t.is_cuda else t.pin_memory() for t in tensors], cpus
    finally:
        os.sched_setaffinity(0, old)


def e2e_steps(args) -> int:
    """Timed steps of the e2e leg: whole c-token cycles (every window of k*c consecutive
    tokens holds exactly k flush tokens of a lockstep batch), at least 8 and about half of
    --steps."""
    c = args.chunk
    return c * max(1, -(-max(8, args.steps // 2) // c))


def time_e2e(wl: Workload, args, ws: int, local: int):
    """Same metric through the public API with HOST buffers: every step copies that
    step's inputs (x, dt, B, C of all layers) from pinned host memory and reads y
    back; copies overlap compute on separate streams, layer by layer.  The timed window is
    whole c-token cycles.  A second run moves the same bytes with no compute (the host
    copy ceiling of this GPU with every rank copying at once)."""
    from nested_ssm_b200 import rot_flat, tiered_state_update
    L, B = wl.L, wl.B
    (hx, hdt, hBC), numa_cpus = pinned_near_gpu([wl.x[0], wl.dt[0], wl.BC[0]], local)
    (hy,), _ = pinned_near_gpu([torch.empty(L, B, H, P, dtype=torch.bfloat16)], local)
    dx = torch.empty_like(wl.x[0])
    ddt = torch.empty_like(wl.dt[0])
    dBC = torch.empty_like(wl.BC[0])
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    comp = torch.cuda.current_stream()
    ev_in = [torch.cuda.Event() for _ in range(L)]
    ev_done = [torch.cuda.Event() for _ in range(L)]
    first = [True]
    h2d = (hx.numel() * hx.element_size() + hdt.numel() * hdt.element_size() + hBC.numel() * hBC.element_size())
    d2h = hy.numel() * hy.element_size()

    def step(compute=True):
        for l in range(L):
            with torch.cuda.stream(s_in):
                if not first[0]:
                    s_in.wait_event(ev_done[l])        # previous step consumed buffer l
                dx[l].copy_(hx[l], non_blocking=True)
                ddt[l].copy_(hdt[l], non_blocking=True)
                dBC[l].copy_(hBC[l], non_blocking=True)
                ev_in[l].record(s_in)
            comp.wait_event(ev_in[l])
            if compute:
                rot_flat(dBC[l], wl.R[l], out=wl.BCr)
                tiered_state_update(wl.pool, l, dx[l], ddt[l], wl.A[l], wl.BCr[:B].view(B, G, N),
                                    wl.BCr[B:].view(B, G, N), wl.D[l], wl.dtb[l], True, wl.slots, -1, wl.y[l],
                                    None, 1e-3)
            ev_done[l].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[l])
                hy[l].copy_(wl.y[l], non_blocking=True)
        first[0] = False

    def timed(K, compute):
        for _ in range(3):
            step(compute)
        torch.cuda.synchronize()
        barrier(ws)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(K):
            step(compute)
        comp.wait_stream(s_out)
        e1.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3 / K
        ms = max_over_ranks(e0.elapsed_time(e1) / K, ws)
        barrier(ws)
        return ms, wall

    K = e2e_steps(args)
    ms, wall = timed(K, True)
    ms_copy, _ = timed(K, False)
    return {"value": round(ws * B / (ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": round(ms, 3), "steps": K,
            "wall_ms_per_step": round(wall, 3),
            "copy_only": {"ms_per_step": round(ms_copy, 3),
                          "gbs_per_gpu": round((h2d + d2h) / (ms_copy / 1e3) / 1e9, 1),
                          "tokens_per_s_ceiling": round(ws * B / (ms_copy / 1e3), 1),
                          "note": "the same host copies with no compute, every rank at once"},
            "bound": "host copies" if ms_copy >= 0.9 * ms else "device compute",
            "pinned_numa_cpus": (f"{numa_cpus[0]}-{numa_cpus[-1]}" if numa_cpus else None)}


def ragged_schedule(steps: int, rows: int, slots: int, seed: int, finish_p: float = 1.0 / 512,
                    admit_p: float = 1.0 / 8, lo: int = 384, init: int = 416, shards: int = 1):
    """Seeded continuous-batching admission process (host side, numpy).

    A batch of `rows` positions holds live sequences (a pool slot each) or padding (-1).
    Every step each live sequence finishes with probability `finish_p` (its slot returns
    to the free list) and each empty position admits a new sequence with probability
    `admit_p`, or always while fewer than `lo` are live.  Returns the per-step slot map
    [steps, rows] and, per step, the slots admitted just before it (fresh state).

    ``shards`` > 1: one global slot space over several GPUs.  Rows and slots split into
    ``shards`` equal contiguous parts (slot shards as ``sharding.slot_range``); a row of part r
    admits only slots of shard r, i.e. a new sequence is routed to a GPU with a free slot and
    stays there; ``lo`` / ``init`` apply per part."""
    import numpy as np
    if rows % shards or slots % shards:
        raise ValueError(f"rows {rows} and slots {slots} must split into {shards} shards")
    rs, ss = rows // shards, slots // shards
    if ss <= rs or not 0 < lo <= init <= rs:
        raise ValueError(f"ragged schedule needs slots > rows >= init >= lo > 0 per shard "
                         f"(slots {ss}, rows {rs}, init {init}, lo {lo})")
    rng = np.random.default_rng(seed)
    free = [list(q * ss + rng.permutation(ss)) for q in range(shards)]
    cur = np.full(rows, -1, dtype=np.int32)
    for q in range(shards):
        for r in rng.choice(rs, init, replace=False):
            cur[q * rs + r] = free[q].pop()
    initial = cur[cur >= 0].copy()
    sched = np.empty((steps, rows), dtype=np.int32)
    admits = []
    for k in range(steps):
        new = []
        if k > 0:
            done = (cur >= 0) & (rng.random(rows) < finish_p)
            for r in np.flatnonzero(done):
                free[r // rs].append(int(cur[r]))
            cur[done] = -1
            admit_draw = rng.random(rows)
            for q in range(shards):
                part = cur[q * rs:(q + 1) * rs]
                empty = np.flatnonzero(part < 0)
                take = empty[admit_draw[q * rs:(q + 1) * rs][empty] < admit_p]
                need = lo - int((part >= 0).sum())
                if need > take.size:
                    take = np.union1d(take, empty[:need])
                for r in take:
                    part[r] = free[q].pop(0)
                    new.append(int(part[r]))
        sched[k] = cur
        admits.append(np.array(new, dtype=np.int32))
    return initial, sched, admits


def time_ragged(args, rank: int, ws: int):
    """Continuous-batching ragged decode (the BASELINE's slot-pool configuration): a pool of
    `--ragged-slots` slots per GPU holding all 27 layers, 384-448 live sequences padded to 448
    rows with slot -1, finishes and admissions every step, and per-slot flush phases (the
    initial sequences start at token counts spread over 0..c-1; admitted ones at 0).  One
    27-layer step is a CUDA graph reading the step's slot map from a device buffer;
    admissions (prefill split of a fresh N(0, 0.1) state into every layer) run between
    steps, outside the timed events.  tokens/s counts live rows only."""
    import numpy as np
    from nested_ssm_b200 import TieredSlotPool, prefill_split, rot_flat, tiered_state_update
    from nested_ssm_b200 import sharding as SH
    dev = torch.device("cuda")
    L, Bm, S, c, K = args.layers, args.batch, args.ragged_slots, args.chunk, args.ragged_steps
    W = max(3, args.warmup)
    # one global schedule (same seed on every rank) over ws*Bm rows and ws*S slots; this rank
    # serves its part of the rows, whose slots all lie in its shard, as local slot ids
    g_initial, g_sched, g_admits = ragged_schedule(W + K, ws * Bm, ws * S, seed=3000, shards=ws)
    lo_s, hi_s = SH.slot_range(ws * S, rank, ws)
    part = g_sched[:, rank * Bm:(rank + 1) * Bm]
    own = SH.owner_of(torch.from_numpy(part[part >= 0]), ws * S, ws)
    assert bool((own == rank).all()), "a row was routed to a GPU that does not own its slot"
    sched = np.where(part >= 0, part - lo_s, -1).astype(np.int32)
    mine = lambda a: (a[(a >= lo_s) & (a < hi_s)] - lo_s).astype(np.int32)   # noqa: E731
    initial = mine(g_initial)
    admits = [mine(a) for a in g_admits]
    gen = torch.Generator(device=dev)
    gen.manual_seed(3000 + rank)
    pool = TieredSlotPool(L, S, H, P, N, G, args.hot, c, args.cold, torch.bfloat16, dev, max_batch=Bm)
    A = [-torch.exp(torch.rand(H, device=dev, generator=gen) * math.log(16.0)) for _ in range(L)]
    D = [torch.randn(H, device=dev, generator=gen) for _ in range(L)]
    dtb = [torch.log(torch.expm1(torch.rand(H, device=dev, generator=gen) * (0.1 - 1e-3) + 1e-3)) for _ in range(L)]
    R = [torch.linalg.qr(torch.randn(G, N, N, device=dev, generator=gen))[0].contiguous() for _ in range(L)]

    def admit(slots_np):
        if slots_np.size == 0:
            return
        sl = torch.from_numpy(slots_np).to(dev)
        for l in range(L):
            st = torch.randn(sl.numel(), H, P, N, device=dev, generator=gen) * math.sqrt(0.1)
            prefill_split(pool, l, st, sl)

    for i in range(0, initial.size, 64):
        admit(initial[i:i + 64])
    ini = torch.from_numpy(initial).long().to(dev)
    pool.t[:, ini, :] = torch.randint(0, c, (ini.numel(), 1), device=dev, generator=gen).int()
    NI = Workload.NI
    x = torch.randn(NI, L, Bm, H, P, device=dev, generator=gen).to(torch.bfloat16)
    dt = torch.randn(NI, L, Bm, H, device=dev, generator=gen).to(torch.bfloat16)
    BC = (torch.randn(NI, L, 2 * Bm, G * N, device=dev, generator=gen) / math.sqrt(N)).to(torch.bfloat16)
    BCr = torch.empty(2 * Bm, G * N, dtype=torch.bfloat16, device=dev)
    y = torch.empty(L, Bm, H, P, dtype=torch.bfloat16, device=dev)
    sched_d = torch.from_numpy(sched).to(dev)
    slots = torch.empty(Bm, dtype=torch.int32, device=dev)

    def one_step(i):
        for l in range(L):
            rot_flat(BC[i, l], R[l], out=BCr)
            tiered_state_update(pool, l, x[i, l], dt[i, l], A[l], BCr[:Bm].view(Bm, G, N), BCr[Bm:].view(Bm, G, N),
                                D[l], dtb[l], True, slots, -1, y[l], None, 1e-3)

    graphs = None
    if not args.no_graph:
        graphs = []
        cap = torch.cuda.Stream()
        slots.copy_(sched_d[0])
        for i in range(NI):
            one_step(i)   # warm every input set once before capture
        torch.cuda.synchronize()
        for i in range(NI):
            g = torch.cuda.CUDAGraph()
            cap.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(cap):
                with torch.cuda.graph(g, stream=cap):
                    one_step(i)
            torch.cuda.current_stream().wait_stream(cap)
            graphs.append(g)
        torch.cuda.synchronize()
        # the warm-up steps above advanced the token counts of the initial sequences; that
        # only shifts their phases
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    live = 0
    for k in range(W + K):
        admit(admits[k])
        slots.copy_(sched_d[k])
        timed = k >= W
        if timed:
            evs[k - W][0].record()
        if graphs is not None:
            graphs[k % NI].replay()
        else:
            one_step(k % NI)
        if timed:
            evs[k - W][1].record()
            live += int((sched[k] >= 0).sum())
    torch.cuda.synchronize()
    pool.check_status()
    tot_ms = sum(a.elapsed_time(b) for a, b in evs)
    ms = max_over_ranks(tot_ms, ws)
    live_all = live
    if ws > 1:
        import torch.distributed as dist
        t = torch.tensor([live], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        live_all = int(t.item())
    ph = (pool.t[0, torch.from_numpy(sched[-1][sched[-1] >= 0]).long().to(dev), 0] % c).bincount(minlength=c)
    del graphs
    return {"tokens_per_s": round(live_all / (ms / 1e3), 1), "ms_per_step": round(ms / K, 4), "steps": K,
            "warmup": W, "live_rows_per_step": round(live / K, 1), "padded_batch": Bm, "slots_per_gpu": S,
            "layers": L, "chunk": c, "n_gpus": ws, "admitted": int(sum(a.size for a in admits[W:])),
            "flush_phase_histogram_last_step": [int(v) for v in ph.tolist()],
            "global_slots": ws * S,
            "config": "continuous batching: finish p=1/512, admit p=1/8 per empty row, >=384 live, "
                      "padded to 448 with slot -1, per-slot flush phases; one global slot space of %d slots "
                      "sharded by slot over %d GPU(s), %d slots x %d layers per GPU (%.1f GB; the "
                      "configuration's 4096 slots x 27 layers per GPU exceed HBM)"
                      % (ws * S, ws, S, L, L * S * bytes_per_slot(args) / 1e9),
            "gpu_launches_per_step": L * 3}


def graph_of_steps(wl: Workload, k0: int):
    """CUDA graph of Workload.NI consecutive steps starting at input set k0."""
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            for k in range(Workload.NI):
                wl.step(k0 + k)
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()
    return g


def time_selfspec(args, rank: int, ws: int, step_ms: float):
    """The self-speculative cycle at the state-op level (what scale/bench_selfspec_e2e.py times
    for the whole model): c hot-only draft tokens (rotation + draft step per layer), one verify
    of the c tokens and the commit of all of them (which flushes: the cycle starts at a chunk
    boundary), over every layer, B sequences, against c ordinary decode steps.  All drafts
    accepted, as the reference's mech(c); a fresh workload so the cycle starts at phase 0."""
    from nested_ssm_b200 import commit_state_update, draft_state_update, verify_state_update
    wl = Workload(args, rank)
    L, B, c, NI = wl.L, wl.B, args.chunk, Workload.NI
    draft = wl.pool.new_draft()
    xs = [torch.stack([wl.x[j % NI, l] for j in range(c)], 1) for l in range(L)]
    dts = [torch.stack([wl.dt[j % NI, l] for j in range(c)], 1) for l in range(L)]
    Bs = [torch.stack([wl.BC[j % NI, l, :B] for j in range(c)], 1).view(B, c, G, N) for l in range(L)]
    Cs = [torch.stack([wl.BC[j % NI, l, B:] for j in range(c)], 1).view(B, c, G, N) for l in range(L)]
    yd = torch.empty(B, H, P, dtype=torch.bfloat16, device="cuda")
    yv = torch.empty(B, c, H, P, dtype=torch.bfloat16, device="cuda")
    accept = torch.full((B,), c, dtype=torch.int32, device="cuda")

    def drafts():
        for j in range(c):
            i = j % NI
            for l in range(L):
                draft_state_update(wl.pool, l, draft[l], wl.x[i, l], wl.dt[i, l], wl.A[l],
                                   wl.BC[i, l, :B].view(B, G, N), wl.BC[i, l, B:].view(B, G, N), wl.D[l], wl.dtb[l],
                                   True, wl.slots, -1, yd, wl.R[l], 1e-3, from_pool=(j == 0))

    def verify():
        for l in range(L):
            verify_state_update(wl.pool, l, xs[l], dts[l], wl.A[l], Bs[l], Cs[l], wl.D[l], wl.dtb[l], True, wl.slots,
                                -1, yv, wl.R[l], 1e-3)

    def commit():
        for l in range(L):
            commit_state_update(wl.pool, l, accept, xs[l], dts[l], wl.A[l], Bs[l], wl.dtb[l], True, wl.slots, -1,
                                wl.R[l], 1e-3)

    for _ in range(2):   # warm-up cycles
        drafts()
        verify()
        commit()
    reps = 4
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4 * reps)]
    barrier(ws)
    torch.cuda.synchronize()
    for r in range(reps):
        ev[4 * r].record()
        drafts()
        ev[4 * r + 1].record()
        verify()
        ev[4 * r + 2].record()
        commit()
        ev[4 * r + 3].record()
    torch.cuda.synchronize()
    d_ms = max_over_ranks(statistics.mean(ev[4 * r].elapsed_time(ev[4 * r + 1]) for r in range(reps)) / c, ws)
    v_ms = max_over_ranks(statistics.mean(ev[4 * r + 1].elapsed_time(ev[4 * r + 2]) for r in range(reps)), ws)
    c_ms = max_over_ranks(statistics.mean(ev[4 * r + 2].elapsed_time(ev[4 * r + 3]) for r in range(reps)), ws)
    barrier(ws)
    wl.pool.check_status()
    del wl, draft, xs, dts, Bs, Cs
    torch.cuda.empty_cache()
    cycle = c * d_ms + v_ms + c_ms
    return {"chunk": c, "draft_tokens": c, "batch_per_gpu": B, "layers": L,
            "draft_ms_per_token": round(d_ms, 4), "verify_ms": round(v_ms, 4), "commit_ms_incl_flush": round(c_ms, 4),
            "cycle_ms": round(cycle, 4), "decode_step_ms": round(step_ms, 4),
            "mech_speedup_all_accepted": round(c * step_ms / cycle, 3),
            "note": "state op only, every layer (rotation included); the model-level gain of self-speculation "
                    "comes from the verify reading the weights once for c tokens, which this leg does not model"}


# The reference's own measurement of this configuration (scale/bench_v4_decode.json: B=256,
# pb=32, c=4, its fp8-cold arm), ms per 27-layer step.
REF_CONFIG1_FP8_MS = 39.0069


def time_config1(args, rank: int, ws: int):
    """B=256 sequences per GPU, 27 layers, c=4, fp8 cold, 256 decode steps
    timed (64 replays of a 4-step CUDA graph: whole c-cycles), inputs resident in HBM."""
    a = argparse.Namespace(**vars(args))
    a.batch, a.chunk, a.cold, a.hot = 256, 4, "fp8", 32
    wl = Workload(a, rank)
    for k in range(3):
        wl.step(k)
    g = graph_of_steps(wl, 3)
    g.replay()
    reps = 256 // Workload.NI
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / (reps * Workload.NI), ws)
    barrier(ws)
    wl.pool.check_status()
    del g, wl
    torch.cuda.empty_cache()
    return {"batch_per_gpu": 256, "layers": 27, "chunk": 4, "cold": "fp8", "steps": reps * Workload.NI,
            "tokens_per_s": round(ws * 256 / (ms / 1e3), 1), "ms_per_step": round(ms, 4),
            "reference_published_ms_per_step": REF_CONFIG1_FP8_MS,
            "speedup_vs_reference_published": round(REF_CONFIG1_FP8_MS / ms, 2)}


REF_DIR = os.path.join(REPO, "baseline", "_ref")


def reference_gpu_leg(batches=(448, 256), pb: int = 32, c: int = 4):
    """The reference's own GPU decode arms, unmodified (``run_point`` of its
    scale/bench_v4_decode.py, installed into baseline/_ref by baseline/install.sh): fla's
    fused recurrent kernel as the fresh op, its v4 arms with fp32 / bf16 / fp8 cold (the fp8
    arm with its own Triton dequant-matvec); the SSU arms need mamba_ssm, absent here.  Runs
    in this process; bench.py starts it in a fresh interpreter."""
    if not os.path.exists(os.path.join(REF_DIR, "bench_v4_decode.py")):
        return {"unavailable": "baseline/_ref/bench_v4_decode.py is not installed (baseline/install.sh)"}
    sys.path.insert(0, REF_DIR)
    import bench_v4_decode as RB   # noqa: E402  (the reference module, unmodified)
    out = {"source": "reference scale/bench_v4_decode.py run_point (unmodified), same box", "points": []}
    for b in batches:
        r = RB.run_point(b, pb, c, "cuda")
        keep = {k: (int(v) if isinstance(v, int) else round(float(v), 4) if math.isfinite(float(v)) else None)
                for k, v in r.items() if k.endswith(("_ms", "_toks")) or k in ("B", "pb", "c")}
        out["points"].append(keep)
        torch.cuda.empty_cache()
    return out


def reference_gpu_leg_isolated(args):
    cmd = [sys.executable, os.path.abspath(__file__), "--reference-gpu-leg-only"]
    env = dict(os.environ)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=1200, env=env)
        return json.loads(out.stdout.strip().splitlines()[-1])
    except (subprocess.TimeoutExpired, ValueError, IndexError) as e:
        return {"unavailable": f"reference GPU leg failed: {type(e).__name__}"}


def multi_gpu_check(args, rank: int, ws: int):
    """Slot-sharded correctness on hardware, outside the timed region: one global slot space
    of ws*64 slots partitioned by slot (sharding.slot_range), a global batch of ws*48 rows with
    a permuted slot map and padded rows.  Every rank serves the rows whose slots it owns
    (sharding.local_batch) for 6 tokens (one flush at c=4; rotation by R on its GPU), y of
    every token is gathered over NCCL (sharding.gather_rows), and rank 0 compares it with its
    own GPU serving the whole global batch alone: the two must be bit-identical."""
    from nested_ssm_b200 import TieredSlotPool, prefill_split, tiered_state_update
    from nested_ssm_b200 import sharding as SH
    dev = torch.device("cuda")
    Sg, Bg, steps, c = 64 * ws, 48 * ws, 6, 4
    gen = torch.Generator().manual_seed(4242)
    slots_g = torch.randperm(Sg, generator=gen)[:Bg].to(torch.int32)
    slots_g[torch.rand(Bg, generator=gen) < 0.05] = -1
    A = -torch.exp(torch.rand(H, generator=gen) * math.log(16.0))
    D = torch.randn(H, generator=gen)
    dtb = torch.log(torch.expm1(torch.rand(H, generator=gen) * (0.1 - 1e-3) + 1e-3))
    R = torch.linalg.qr(torch.randn(G, N, N, generator=gen))[0].contiguous()
    xs = torch.randn(steps, Bg, H, P, generator=gen).to(torch.bfloat16)
    dts = torch.randn(steps, Bg, H, generator=gen).to(torch.bfloat16)
    Bs = (torch.randn(steps, Bg, G, N, generator=gen) / math.sqrt(N)).to(torch.bfloat16)
    Cs = (torch.randn(steps, Bg, G, N, generator=gen) / math.sqrt(N)).to(torch.bfloat16)
    A, D, dtb, R = A.to(dev), D.to(dev), dtb.to(dev), R.to(dev)

    def fill(pool, lo, hi):
        """Prefill global slots [lo, hi) into pool slots 0.. from one seeded global stream."""
        g = torch.Generator(device=dev).manual_seed(99)
        for s0 in range(0, Sg, 64):
            st = torch.randn(64, H, P, N, device=dev, generator=g) * math.sqrt(0.1)
            sel = [i for i in range(64) if lo <= s0 + i < hi]
            if sel:
                loc = torch.tensor([s0 + i - lo for i in sel], dtype=torch.int32, device=dev)
                prefill_split(pool, 0, st[sel].contiguous(), loc)

    lo, hi = SH.slot_range(Sg, rank, ws)
    pool = TieredSlotPool(1, hi - lo, H, P, N, G, args.hot, c, args.cold, torch.bfloat16, dev, max_batch=Bg)
    fill(pool, lo, hi)
    rows, lsl = SH.local_batch(slots_g, rank, ws, Sg)
    gathered = []
    for k in range(steps):
        y = torch.zeros(rows.numel(), H, P, dtype=torch.bfloat16, device=dev)
        if rows.numel():
            tiered_state_update(pool, 0, xs[k][rows].to(dev), dts[k][rows].to(dev), A, Bs[k][rows].to(dev),
                                Cs[k][rows].to(dev), D, dtb, True, lsl.to(dev), -1, y, R, 1e-3)
        gathered.append(SH.gather_rows(y, rows.to(dev), Bg))
    torch.cuda.synchronize()
    pool.check_status()
    n_rows = int(rows.numel())
    del pool
    if rank != 0:
        return None
    single = TieredSlotPool(1, Sg, H, P, N, G, args.hot, c, args.cold, torch.bfloat16, dev, max_batch=Bg)
    fill(single, 0, Sg)
    worst, equal = 0.0, True
    for k in range(steps):
        y1 = torch.zeros(Bg, H, P, dtype=torch.bfloat16, device=dev)
        tiered_state_update(single, 0, xs[k].to(dev), dts[k].to(dev), A, Bs[k].to(dev), Cs[k].to(dev), D, dtb,
                            True, slots_g.to(dev), -1, y1, R, 1e-3)
        equal &= bool(torch.equal(y1, gathered[k]))
        worst = max(worst, float((y1.float() - gathered[k].float()).abs().max()))
    single.check_status()
    del single
    torch.cuda.empty_cache()
    return {"pass": equal, "max_abs_diff": worst, "global_slots": Sg, "global_batch": Bg,
            "padded_rows": int((slots_g < 0).sum()), "rows_on_rank0": n_rows, "steps": steps,
            "check": "y of every token, slot-sharded over the ranks and gathered over NCCL, "
                     "bit-identical to one GPU serving the whole global batch"}


NEMOTRON_9B_LAYOUT = "M-M-M-MM-M-M-M*-M-M-M*-M-M-M-M*-M-M-M-M*-M-MM-M-M-M-M-M-"   # the published 9B-v2 layout


def nemotron_h_9b(device="cuda", chunk_size=8):
    """The BASELINE's end-to-end architecture (Nemotron-H 9B), random init, bf16: hidden 4480,
    56 layers = 27 Mamba2 (128 heads x 80, d_state 128, 8 groups, conv 4) + 4 GQA attention
    (40 q / 8 kv heads of 128) + 25 ReLU^2 MLP (intermediate 15680), vocab 131072, weights
    ~N(0, 0.02).  transformers 5.5's NemotronH has no dense-MLP block type ("-" in the published
    layout), so those blocks are built as NemotronHMLP under the "moe" type, whose block forward is
    the same plain mixer(hidden) call and whose attention mask is None.  ``chunk_size`` is the
    prefill scan's chunk, which the decode does not use: the model's own naive prefill pads the
    prompt to whole chunks and holds fp32 products of (batch, chunks, chunk, chunk, heads, d_state)
    and of (batch, padded prompt, heads, headdim, d_state) -- 1.9 GB and 19 GB at B = 448 with an
    8-token prompt and chunk 8, but 481 GB for the first at the published chunk 128."""
    from transformers import NemotronHConfig, NemotronHForCausalLM
    from transformers.models.nemotron_h import modeling_nemotron_h as MH
    layout = NEMOTRON_9B_LAYOUT
    kinds = {"M": "mamba", "*": "attention", "-": "moe"}
    cfg = NemotronHConfig(hidden_size=4480, layers_block_type=[kinds[ch] for ch in layout],
                          num_hidden_layers=len(layout), mamba_num_heads=128, mamba_head_dim=80,
                          ssm_state_size=128, n_groups=8, conv_kernel=4, expand=2, intermediate_size=15680,
                          mlp_hidden_act="relu2", num_attention_heads=40, num_key_value_heads=8, head_dim=128,
                          vocab_size=131072, chunk_size=chunk_size, initializer_range=0.02)
    saved = MH.MIXER_TYPES["moe"]
    MH.MIXER_TYPES["moe"] = lambda config, layer_idx=None: MH.NemotronHMLP(config)
    try:
        with torch.device(device):
            model = NemotronHForCausalLM(cfg)
    finally:
        MH.MIXER_TYPES["moe"] = saved
    return model.to(torch.bfloat16).eval()


def model_e2e(args, device="cuda", build=None):
    """Reduced BASELINE config 4 on one GPU: decode tokens/s of a random-init Nemotron-H 9B (bf16,
    weights ~N(0, 0.02)) with seeded per-group rotations (the reference's ActRotMask around every
    mixer's activation), B sequences of `--model-prompt` random tokens, `--model-gen` greedy
    tokens through transformers' generate.  Decode time = generate(gen + 1) - generate(1), so the
    prefill cancels; the prefill is the model's own in every arm (this image has no mamba_ssm, and
    the lean chunk-scan prefill wants chunk 128).  Arms on the same model and box: `ours`
    (nested_ssm_b200.hf.install: conv step, tiered step with the fused norm; fp8 cold, c = 4),
    `reference` (the reference's own scale/v4_native_decode.install, unmodified from baseline/_ref;
    bf16 cold, its default), `hf` (transformers' own decode over the fresh full state)."""
    if not os.path.exists(os.path.join(REF_DIR, "nemotron_retrofit.py")):
        return {"unavailable": "baseline/_ref is not installed (baseline/install.sh): the rotation wrapper is the "
                               "reference's ActRotMask"}
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import nemotron_retrofit as NR   # noqa: E402  (the reference's modules, unmodified)
    import v4_native_decode as V4   # noqa: E402
    build = build or nemotron_h_9b
    Bm, T, K = args.model_batch, args.model_prompt, args.model_gen
    out = {"config": {"workload": "reduced BASELINE config 4: random-init Nemotron-H 9B architecture, bf16, "
                                  f"B={Bm}, prompt {T} random tokens, {K} greedy decode tokens "
                                  "(the config's 4096 / 512 reduced), one GPU, decode = generate(K+1) - generate(1)",
                      "batch": Bm, "prompt": T, "gen": K}, "arms": {}}
    for arm in [a for a in args.model_arms.split(",") if a]:
        torch.manual_seed(0)
        model = build(device)
        g = torch.Generator(device=device).manual_seed(1)
        for m in model.modules():
            if type(m).__name__ == "NemotronHMamba2Mixer":
                act = NR.ActRotMask(m.act, m.intermediate_size, m.n_groups, m.ssm_state_size).to(device)
                q = torch.linalg.qr(torch.randn(m.n_groups, m.ssm_state_size, m.ssm_state_size, device=device,
                                                generator=g))[0]
                act.R.data.copy_(q)
                m.act = act
        if arm == "ours":
            from nested_ssm_b200 import hf as HF
            HF.install(model, pb=32, c=4, cold="fp8")
        elif arm == "reference":
            V4.install(model, pb=32, c=4)
            for m in model.modules():
                if hasattr(m, "v4cfg"):
                    m.v4cfg["lean_prefill"] = 0   # its lean prefill imports mamba_ssm, absent here
        ids = torch.randint(1000, 30000, (Bm, T), device=device, generator=g)
        gk = dict(do_sample=False, pad_token_id=0, eos_token_id=None)
        sync = torch.cuda.synchronize if device == "cuda" else (lambda: None)

        def gen(n):
            sync()
            t0 = time.perf_counter()
            with torch.no_grad():
                toks = model.generate(ids, max_new_tokens=n, **gk)
            sync()
            return time.perf_counter() - t0, toks

        try:
            gen(2)                                   # warm-up (kernels, allocator)
            (t1, _), (tk, toks) = gen(1), gen(K + 1)
            dec = (tk - t1) / K
            res = {"decode_ms_per_token": round(dec * 1e3, 2), "decode_tokens_per_s": round(Bm / dec, 1),
                   "prefill_s": round(t1, 3), "tokens_crc": int(toks[:, T:].to(torch.int64).sum())}
            if device == "cuda":
                res["peak_gb"] = round(torch.cuda.max_memory_allocated() / 1e9, 1)
            out["arms"][arm] = res
        except torch.cuda.OutOfMemoryError as e:
            out["arms"][arm] = {"unavailable": f"out of memory: {str(e)[:160]}"}
        del model
        if device == "cuda":
            torch.cuda.empty_cache()
            torch.cuda.reset_peak_memory_stats()
    return out


# --------------------------------------------------------------------------
# serving-engine decode: vLLM 0.22, stock against the tiered hook (reduced BASELINE config 4)
# --------------------------------------------------------------------------
def vllm_model_dir(root: str) -> str:
    """A model directory holding only the Nemotron-H 9B config (vLLM's own NemotronH config
    class reads the "-" MLP layers); the weights are vLLM's dummy initialisation."""
    d = os.path.join(root, "nemotron_h_9b")
    os.makedirs(d, exist_ok=True)
    cfg = {"architectures": ["NemotronHForCausalLM"], "model_type": "nemotron_h", "vocab_size": 131072,
           "hidden_size": 4480, "intermediate_size": 15680, "num_hidden_layers": len(NEMOTRON_9B_LAYOUT),
           "hybrid_override_pattern": NEMOTRON_9B_LAYOUT, "num_attention_heads": 40, "head_dim": 128,
           "num_key_value_heads": 8, "mlp_hidden_act": "relu2", "ssm_state_size": 128, "mamba_num_heads": 128,
           "mamba_n_groups": 8, "mamba_head_dim": 80, "mamba_d_conv": 4, "mamba_expand": 2,
           "mamba_chunk_size": 128, "max_position_embeddings": 8192, "torch_dtype": "bfloat16",
           "initializer_range": 0.02, "layer_norm_epsilon": 1e-5, "tie_word_embeddings": False,
           "bos_token_id": 1, "eos_token_id": 2, "pad_token_id": 0}
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    return d


# vLLM's dummy weights never pass through load_weights (where the hook applies its checkpoint),
# so the shadow copy applies it at the end of NemotronHForCausalLM.__init__ as well
_VLLM_INIT_ANCHOR = ("        self.make_empty_intermediate_tensors = (\n"
                     "            self.model.make_empty_intermediate_tensors\n"
                     "        )\n")
_VLLM_INIT_TEXT = ("        from nested_ssm_b200 import vllm_hook as _nssm\n"
                   "        _nssm.apply_ckpt(self)  # [nested_ssm] dummy weights: load_weights is not called\n")


def vllm_shadow(root: str) -> str:
    """A shadow of the installed vllm package under ``root`` (directories, file symlinks) whose
    mamba_mixer2.py and nemotron_h.py are patched copies (the hook's five anchors and the init
    call); returns the directory to put first on PYTHONPATH.  The installed package is not
    modified."""
    import importlib.util
    import shutil
    from nested_ssm_b200 import vllm_hook as VH
    src = os.path.dirname(importlib.util.find_spec("vllm").origin)
    top = os.path.join(root, "shadow")
    dst = os.path.join(top, "vllm")
    if not os.path.isdir(dst):
        os.makedirs(top, exist_ok=True)
        subprocess.run(["cp", "-rs", src, dst], check=True)
        for rel in (VH.MIXER, VH.NEMOTRON):
            path = os.path.join(dst, rel)
            os.remove(path)
            shutil.copyfile(os.path.join(src, rel), path)
        VH.install(dst)
        path = os.path.join(dst, VH.NEMOTRON)
        with open(path) as f:
            text, _ = VH.patch_source(f.read(), "after", _VLLM_INIT_ANCHOR, _VLLM_INIT_TEXT, VH.NEMOTRON)
        with open(path, "w") as f:
            f.write(text)
    return top


def vllm_rotation_ckpt(root: str, identity: bool = False, mixers: int = 27, G_: int = 8, N_: int = 128) -> str:
    """Seeded orthogonal rotations (or identities) in the hook's checkpoint format {i: R_i [G, N, N]}."""
    path = os.path.join(root, "rot_identity.pt" if identity else "rot.pt")
    g = torch.Generator().manual_seed(7)
    torch.save({i: (torch.eye(N_).repeat(G_, 1, 1) if identity
                    else torch.linalg.qr(torch.randn(G_, N_, N_, generator=g))[0].contiguous()) for i in range(mixers)},
               path)
    return path


def vllm_e2e(args):
    """Reduced BASELINE config 4 in a serving engine: vLLM 0.22 (CUDA-graph decode, its own
    fused Mamba2 kernels) on a dummy-weight Nemotron-H 9B, B sequences of `--model-prompt`
    random tokens, `--model-gen` greedy tokens; decode = generate(gen + 1) - generate(1).
    Arms: `vllm` (stock: fresh fp32 full state, vLLM's selective_state_update), `ours` (the same
    engine with the tiered decode installed by nested_ssm_b200.vllm_hook: rotations from a
    seeded checkpoint, fp8 cold, c = 4, the stale readout) and `ours_exact` (identity rotations,
    fp32 cold, the exact rank-c correction readout: the tiered op's exact configuration, whose
    greedy tokens are compared with the stock arm's as a check that the hook runs correctly
    inside the engine; with `--vllm-reinit` the weights make the tokens depend on the state).  Each arm runs in its own
    process; both use an fp32 SSM cache (mamba_ssm_cache_dtype), the reference's setting."""
    root = tempfile.mkdtemp(prefix="nssm_vllm_")
    model = vllm_model_dir(root)
    out = {"config": {"workload": f"reduced BASELINE config 4 in vLLM 0.22: dummy-weight Nemotron-H 9B, bf16, "
                                  f"B={args.model_batch}, prompt {args.model_prompt}, {args.model_gen} greedy tokens, "
                                  "one GPU, decode = generate(K+1) - generate(1)",
                      "batch": args.model_batch, "prompt": args.model_prompt, "gen": args.model_gen,
                      "gpu_memory_utilization": {"vllm": args.vllm_mem, "ours": args.vllm_mem_ours}}, "arms": {}}
    for arm in [a for a in args.vllm_arms.split(",") if a]:
        env = dict(os.environ)
        env["PYTHONPATH"] = REPO + (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
        base = arm[:-len("_eager")] if arm.endswith("_eager") else arm   # _eager: no CUDA graphs
        if base == "ours_fresh":   # the hook in fresh mode, identity R: vLLM's own update, the hook's copies
            env["PYTHONPATH"] = vllm_shadow(root) + os.pathsep + env["PYTHONPATH"]
            env.update(NESTED_SSM_CKPT=vllm_rotation_ckpt(root, identity=True), NESTED_SSM_MODE="fresh")
        if base in ("ours", "ours_exact"):
            exact = base == "ours_exact"
            env["PYTHONPATH"] = vllm_shadow(root) + os.pathsep + env["PYTHONPATH"]
            env.update(NESTED_SSM_CKPT=vllm_rotation_ckpt(root, identity=exact), NESTED_SSM_MODE="v4",
                       NESTED_SSM_PB="32", NESTED_SSM_C="4", NESTED_SSM_COLD="fp32" if exact else "fp8",
                       NESTED_SSM_READOUT="corr" if exact else "stale")
        cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--vllm-arm", arm, "--vllm-model", model,
               "--vllm-tokens", os.path.join(root, f"tokens_{arm}.pt"),
               "--model-batch", str(args.model_batch), "--model-prompt", str(args.model_prompt),
               "--model-gen", str(args.model_gen),
               "--vllm-mem", str(args.vllm_mem if arm.startswith("vllm") else args.vllm_mem_ours),
               "--vllm-blocks", str(args.vllm_blocks)] + (["--vllm-reinit"] if args.vllm_reinit else []) + \
              (["--vllm-eager"] if arm.endswith("_eager") else [])
        r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=1800)
        line = next((ln for ln in reversed(r.stdout.splitlines()) if ln.startswith("{")), None)
        text = (r.stderr or "") + (r.stdout or "")
        if r.returncode != 0 or line is None:
            errs = [ln.strip()[-300:] for ln in text.splitlines() if "Error" in ln or "error" in ln][:6]
            out["arms"][arm] = {"unavailable": f"exit {r.returncode}", "errors": errs, "tail": text[-400:]}
            continue
        res = json.loads(line)
        keys = ("[nested_ssm]", "KV cache size", "Maximum concurrency", "Graph capturing finished", "cudagraph_mode")
        res["log"] = [ln.strip()[-200:] for ln in text.splitlines() if any(k in ln for k in keys)][:8]
        import re
        m = re.search(r"Maximum concurrency for (\d+) tokens per request: ([\d.]+)x", text)
        if m:   # the per-token rate assumes all B rows decode together
            res["max_concurrency"] = float(m.group(2))
            res["all_rows_concurrent"] = float(m.group(2)) >= args.model_batch
        out["arms"][arm] = res
    ref = os.path.join(root, "tokens_vllm.pt")
    for arm in [a for a in out["arms"] if a != "vllm"]:   # e.g. vllm_eager: stock against stock
        mine = os.path.join(root, f"tokens_{arm}.pt")
        if arm in out["arms"] and os.path.exists(ref) and os.path.exists(mine):
            ra, rb = torch.load(ref), torch.load(mine)
            a, b = ra["tokens"], rb["tokens"]
            o = out["arms"][arm]
            o["greedy_tokens_equal_to_stock"] = round(float((a == b).float().mean()), 4)
            o["first_token_equal_to_stock"] = round(float((a[:, 0] == b[:, 0]).float().mean()), 4)
            # while both arms have produced the same tokens, they score the same contexts: the
            # sampled token's log-probability then measures how far the decode outputs differ
            same = torch.cumprod((a == b).to(torch.int32), dim=1).bool()
            if ra["logprobs"] is not None and rb["logprobs"] is not None and bool(same[:, 1:].any()):
                d = (ra["logprobs"] - rb["logprobs"]).abs()[:, 1:][same[:, 1:]]
                o["decode_logprob_abs_diff_on_common_prefix"] = {"max": round(float(d.max()), 5),
                                                                 "mean": round(float(d.mean()), 6),
                                                                 "tokens": int(d.numel())}
            div = torch.where((~same).any(1), (~same).float().argmax(1), torch.full_like(a[:, 0], a.shape[1]))
            o["first_divergence_mean_position"] = round(float(div.float().mean()), 2)
    return out


def _vllm_reinit(model):
    """Seeded weights with the BASELINE's distributions in place of vLLM's dummy ones (which are
    so small that every layer's output vanishes next to the embedding, so the greedy tokens would
    not depend on the Mamba state): N(0, 0.02) matrices, A = -exp(U(0, ln 16)), dt_bias =
    softplus^-1(U(1e-3, 0.1)), D and norm weights 1, biases 0.  Each parameter's draw is seeded by
    its name, so every arm gets the same model.  The hook's cached fp32 copies of A, D and dt_bias
    are refreshed in place."""
    import math as m_
    import zlib
    with torch.inference_mode():   # the hook's caches were made inside vLLM's inference mode
        for name, p in sorted(model.named_parameters()):
            g = torch.Generator(device=p.device)
            g.manual_seed(zlib.crc32(name.encode()))
            if name.endswith(".A"):
                p.copy_(-torch.exp(torch.rand(p.shape, generator=g, device=p.device) * m_.log(16.0)))
            elif name.endswith("dt_bias"):
                u = torch.rand(p.shape, generator=g, device=p.device) * (0.1 - 1e-3) + 1e-3
                p.copy_(torch.log(torch.expm1(u)))
            elif name.endswith(".D") or "norm" in name:
                p.fill_(1.0)
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.copy_(torch.randn(p.shape, generator=g, device=p.device, dtype=torch.float32) * 0.02)
        for mod in model.modules():
            st = getattr(mod, "nssm", None)
            if isinstance(st, dict) and "A" in st:
                st["A"].copy_(mod.A.detach().float().reshape(-1))
                st["D"].copy_(mod.D.detach().float().reshape(-1))
                st["dt_bias"].copy_(mod.dt_bias.detach().float().reshape(-1))
    return True


def _vllm_pool_stats(model):
    """The tiered pools' bookkeeping after a run (hooked arms): how many mixers hold a pool, the
    largest token count t, and the pools' status words."""
    n, tmax, status = 0, 0, 0
    for mod in model.modules():
        st = getattr(mod, "nssm", None)
        if isinstance(st, dict) and st.get("pool") is not None:
            n += 1
            tmax = max(tmax, int(st["pool"].t.max()))
            status |= int(st["pool"].status.item())
    return {"mixers_with_pool": n, "t_max": tmax, "status": status}


def vllm_arm(args):
    """One arm of vllm_e2e, in its own process (the parent chose the vllm package by PYTHONPATH)."""
    import vllm
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt
    from vllm.transformers_utils.config import _CONFIG_REGISTRY
    # transformers' own NemotronH config has no dense-MLP ("-") layers; vLLM ships one that does
    _CONFIG_REGISTRY["nemotron_h"] = "NemotronHConfig"
    B, T, K = args.model_batch, args.model_prompt, args.model_gen
    if args.vllm_reinit:   # apply_model sends the function to the engine's worker process
        os.environ["VLLM_ALLOW_INSECURE_SERIALIZATION"] = "1"
    kw = dict(model=args.vllm_model, skip_tokenizer_init=True, load_format="dummy", dtype="bfloat16",
              max_num_seqs=B, max_model_len=T + K + 16, gpu_memory_utilization=args.vllm_mem,
              enable_prefix_caching=False, seed=0, mamba_ssm_cache_dtype="float32")
    if args.vllm_blocks:
        kw["num_gpu_blocks_override"] = args.vllm_blocks
    if args.vllm_eager:
        kw["enforce_eager"] = True
    llm = LLM(**kw)
    if args.vllm_reinit:
        llm.apply_model(_vllm_reinit)
    g = torch.Generator().manual_seed(1)
    prompts = [TokensPrompt(prompt_token_ids=r) for r in torch.randint(1000, 30000, (B, T), generator=g).tolist()]

    def run(n):
        sp = SamplingParams(max_tokens=n, ignore_eos=True, temperature=0.0, detokenize=False, logprobs=0)
        t0 = time.perf_counter()
        outs = llm.generate(prompts, sp, use_tqdm=False)
        return time.perf_counter() - t0, outs

    run(4)   # warm-up
    t1, _ = run(1)
    tk, outs = run(K + 1)
    dec = (tk - t1) / K
    toks = torch.tensor([list(o.outputs[0].token_ids) for o in outs])   # LLM.generate keeps prompt order
    lps = torch.tensor([[float(d[t].logprob) for d, t in zip(o.outputs[0].logprobs, o.outputs[0].token_ids)]
                        for o in outs]) if outs[0].outputs[0].logprobs else None
    if args.vllm_tokens:
        torch.save({"tokens": toks, "logprobs": lps}, args.vllm_tokens)
    pools = None
    if os.environ.get("NESTED_SSM_MODE") == "v4" and os.environ.get("VLLM_ALLOW_INSECURE_SERIALIZATION") == "1":
        pools = llm.apply_model(_vllm_pool_stats)
    res = {"decode_ms_per_token": round(dec * 1e3, 2), "decode_tokens_per_s": round(B / dec, 1),
           "prefill_plus_one_s": round(t1, 3), "tokens": int(toks.numel()), "vllm": vllm.__version__,
           "vllm_path": os.path.dirname(vllm.__file__),
           "tiered_hook": os.environ.get("NESTED_SSM_MODE") == "v4",
           "cold": os.environ.get("NESTED_SSM_COLD") if os.environ.get("NESTED_SSM_MODE") == "v4" else None,
           "readout": os.environ.get("NESTED_SSM_READOUT") if os.environ.get("NESTED_SSM_MODE") == "v4" else None,
           "pools": pools}
    print(json.dumps(res), flush=True)
    return 0


# --------------------------------------------------------------------------
# CPU legs (the oracle port -- the reference's own path is Python/torch)
# --------------------------------------------------------------------------
def cpu_sample(args, batch: int, steps: int, warmup: int, threads: int):
    """Time the CPU oracle (tiered replay semantics, torch eager) on `batch` sequences
    x all layers; returns tokens/s and a description."""
    import oracle as O
    torch.set_num_threads(threads)
    L = args.layers
    cold = {"fp8": O.FP8, "bf16": torch.bfloat16, "fp32": torch.float32}[args.cold]
    prms = O.make_params(H, G, N, seed=0, layers=L)
    pools = []
    for l in range(L):
        pool = O.TieredPoolRef(batch, H, P, N, G, args.hot, args.chunk, cold, torch.bfloat16)
        O.prefill_split(pool, torch.arange(batch), torch.randn(batch, H, P, N) * math.sqrt(0.1))
        pools.append(pool)
    xs, dts, Bs, Cs = O.make_inputs(batch, H, P, G, N, args.chunk, seed=0)
    slots = torch.arange(batch)

    def step(k):
        i = k % args.chunk
        for l in range(L):
            prm = prms[l]
            Br = O.rot_flat(Bs[i].reshape(batch, -1), prm["R"]).reshape(batch, G, N)
            Cr = O.rot_flat(Cs[i].reshape(batch, -1), prm["R"]).reshape(batch, G, N)
            O.tiered_step(pools[l], slots, xs[i], dts[i], Br, Cr, prm["A"], prm["D"], prm["dt_bias"], 1e-3)

    for k in range(warmup):
        step(k)
    t0 = time.perf_counter()
    times = []
    for k in range(steps):
        s0 = time.perf_counter()
        step(k)
        times.append(time.perf_counter() - s0)
    el = time.perf_counter() - t0
    return {"tokens_per_s": batch * steps / el, "step_s": times}


def host_threads() -> int:
    """Cores this process may run on (its CPU affinity; containers often allow fewer than
    os.cpu_count() reports, and more torch threads than cores only slows the CPU legs)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_baseline_leg_isolated(args):
    """The CPU leg in a fresh interpreter: the bench process, after its GPU legs, runs the
    same torch CPU code tens of times slower than a clean process does."""
    cmd = [sys.executable, os.path.abspath(__file__), "--cpu-leg-only", "--layers", str(args.layers),
           "--chunk", str(args.chunk), "--hot", str(args.hot), "--cold", args.cold,
           "--cpu-sample-batch", str(args.cpu_sample_batch)]
    env = dict(os.environ)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
        return json.loads(out.stdout.strip().splitlines()[-1])
    except (subprocess.TimeoutExpired, ValueError, IndexError) as e:
        return {"value": None, "unit": "tokens/s", "error": f"cpu leg failed: {type(e).__name__}"}


def cpu_baseline_leg(args):
    threads = host_threads()
    r = cpu_sample(args, args.cpu_sample_batch, args.chunk, 1, threads)
    return {"value": round(r["tokens_per_s"], 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"oracle (torch eager, {threads} threads): B={args.cpu_sample_batch} sequences x "
                      f"{args.layers} layers x {args.chunk} steps (one flush cycle), same shapes/dtypes"}


def run_reference(args):
    """--impl reference: the reference's CPU path (the oracle port; the reference is
    Python with no compiled CPU code) on the host cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = host_threads()
    batch = args.cpu_sample_batch
    r = cpu_sample(args, batch, max(1, args.steps), max(0, min(args.warmup, 1)), threads)
    v = round(r["tokens_per_s"], 3)
    ms = statistics.mean(r["step_s"]) * 1e3
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.cold + "-cold/fp32-hot", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"tiered c={args.chunk} {args.cold}-cold hot={args.hot}, {args.layers} layers, "
                                   f"sampled at B={batch} (CPU)", "batch": batch, "layers": args.layers},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"B={batch} sequences x {args.layers} layers per step, torch eager CPU"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------
def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.cpu_leg_only:
        print(json.dumps(cpu_baseline_leg(args)), flush=True)
        return 0
    if args.reference_gpu_leg_only:
        print(json.dumps(reference_gpu_leg()), flush=True)
        return 0
    if args.vllm_arm:
        return vllm_arm(args)
    if args.vllm_e2e:
        print(json.dumps({"vllm_e2e": vllm_e2e(args)}), flush=True)
        return 0
    if args.model_e2e:
        if not torch.cuda.is_available():
            raise SystemExit("bench.py --model-e2e needs a CUDA device")
        print(json.dumps({"model_e2e": model_e2e(args)}), flush=True)
        return 0
    rank, ws, local = dist_init()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    import nested_ssm_b200  # noqa: F401  (fails loudly if the library is missing)
    if args.prefill_only:
        pf = time_prefill(args, rank, ws)
        if rank == 0:
            print(json.dumps({"prefill_scan": pf}), flush=True)
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return 0
    wl = Workload(args, rank)
    L, B, K, W = wl.L, wl.B, args.steps, max(3, args.warmup)

    # A CUDA graph holds Workload.NI consecutive steps (every layer: rotation then the
    # tiered update); the flush decision is taken on the device from the slots' token
    # counts, so replays stay exact.
    NI = Workload.NI
    evs = [[[torch.cuda.Event(enable_timing=True, external=True) for _ in range(3)] for _ in range(L)]
           for _ in range(NI)]
    for k in range(W):
        wl.step(k)
    torch.cuda.synchronize()
    # Two graphs of the same NI steps: the timed one holds only the kernels; the other adds
    # event-record nodes around every layer's launches for the per-kernel breakdown (those
    # nodes are measurement, not work, so they stay out of the timed region).
    graph = graph_ev = None
    if not args.no_graph:
        cap = torch.cuda.Stream()
        graphs = []
        for with_ev in (False, True):
            cap.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(cap):
                with torch.cuda.graph(g, stream=cap):
                    for k in range(NI):
                        wl.step(W + k, evs[k] if with_ev else None)
            torch.cuda.current_stream().wait_stream(cap)
            graphs.append(g)
        graph, graph_ev = graphs
        torch.cuda.synchronize()
        # (capture did not execute the kernels)
    reps = max(1, (K + NI - 1) // NI)
    K = reps * NI

    def run_cycle(k0, events=False):
        if graph is not None:
            (graph_ev if events else graph).replay()
        else:
            for k in range(NI):
                wl.step(k0 + k, evs[k] if events else None)

    run_cycle(0)   # warm both graphs
    run_cycle(0, events=True)
    barrier(ws)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for r in range(reps):
        run_cycle(r * NI)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / K, ws)
    barrier(ws)

    # kernel durations over whole c-cycles (flush and non-flush launches), from the
    # event-record nodes of further replays
    kd_all, rd_all = [], []
    for r in range(max(1, (args.chunk + NI - 1) // NI)):
        run_cycle(0, events=True)
        torch.cuda.synchronize()
        for k in range(NI):
            kd_all += [evs[k][l][1].elapsed_time(evs[k][l][2]) for l in range(L)]
            rd_all += [evs[k][l][0].elapsed_time(evs[k][l][1]) for l in range(L)]
    value = ws * B / (ms / 1e3)

    peak, peak_kind = load_peaks()
    bps = step_bytes_per_seq(args.chunk, args.hot, args.cold)
    kms = statistics.mean(kd_all) if kd_all else None
    roof = None
    if kms:
        achieved = B * bps / (kms / 1e3) / 1e9
        tr = load_traffic()
        traffic = None
        if tr and tr.get("workload") == f"B{B}_c{args.chunk}_{args.cold}_pb{args.hot}":
            traffic = tr.get("bytes_per_launch")
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                "kernel": "tiered state update (STEP + FLUSH persistent kernels)", "kernel_ms_avg": round(kms, 4),
                "bytes_per_launch": int(B * bps), "reference_model_bytes_per_launch": int(B * reference_model_bytes_per_seq(args.chunk)),
                "rotation_ms_avg": round(statistics.mean(rd_all), 4) if rd_all else None,
                "kernel_ms_by_step": [round(statistics.mean(kd_all[i * L:(i + 1) * L]), 4)
                                      for i in range(len(kd_all) // L)],
                "step_gbs_incl_rotation": round(L * B * bps / (ms / 1e3) / 1e9, 1)}

    e2e = None if args.no_e2e else time_e2e(wl, args, ws, local)
    del wl
    torch.cuda.empty_cache()
    fresh = None if args.no_fresh else time_fresh(args, rank, ws)
    conv = None if args.no_conv else time_conv(args, rank, ws)
    prefill = None if args.no_prefill else time_prefill(args, rank, ws)
    torch.cuda.empty_cache()
    ragged = None if args.no_ragged else time_ragged(args, rank, ws)
    torch.cuda.empty_cache()
    config1 = None if args.no_config1 else time_config1(args, rank, ws)
    torch.cuda.empty_cache()
    selfspec = None if args.no_selfspec else time_selfspec(args, rank, ws, ms)
    mcheck = None if (ws == 1 or args.no_multi_gpu_check) else multi_gpu_check(args, rank, ws)
    ref_gpu = None
    if rank == 0 and ws == 1 and not args.no_reference_gpu:
        torch.cuda.empty_cache()
        ref_gpu = reference_gpu_leg_isolated(args)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_baseline_leg_isolated(args)

    if rank == 0:
        # vs_baseline: against the reference's own fp8-cold arm measured on this box in this run
        # when that leg ran, else against its published number (other box)
        ref_same = None
        if ref_gpu and ref_gpu.get("points"):
            ref_same = next((p_.get("v4fp8_toks") for p_ in ref_gpu["points"] if p_.get("B") == B), None)
        base_toks = ref_same if ref_same else REF_PUBLISHED_TOKS
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": ws, "steps": K,
            "warmup": W, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": round(value / (ws * base_toks), 3),
            "vs_baseline_denominator": ("reference fp8-cold arm, same box, this run (tokens/s per GPU): %.1f"
                                        % ref_same) if ref_same else
                                       ("reference published fp8-cold arm (other box): %.1f tokens/s"
                                        % REF_PUBLISHED_TOKS),
            "dtype": f"{args.cold}-cold/fp32-hot (bf16 io)", "data": "synthetic",
            "config": {"workload": f"tiered c={args.chunk} {args.cold}-cold hot={args.hot}, B={B}/GPU, "
                                   f"{L} layers, H={H} P={P} N={N} G={G}",
                       "batch_per_gpu": B, "layers": L, "chunk": args.chunk, "hot": args.hot, "cold": args.cold,
                       "parallelism": f"slot-sharded x{ws} (no collective)",
                       "l2": "inputs larger than L2 (tiered pool %.1f GB/GPU)" % (L * B * bytes_per_slot(args) / 1e9),
                       "cuda_graph": not args.no_graph},
            "gpu_launches": K * L * 3,   # per layer: rotation, STEP, FLUSH
            "roofline": roof,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "fresh_control": fresh,
            "speedup_vs_fresh": round(value / fresh["tokens_per_s"], 3) if fresh else None,
            "conv_step": conv,
            "prefill_scan": prefill,
            "ragged": ragged,
            "config1": config1,
            "selfspec": selfspec,
            "reference_gpu": ref_gpu,
            "multi_gpu_check": mcheck,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def bytes_per_slot(args) -> float:
    s = {"fp8": 1, "bf16": 2, "fp32": 4}[args.cold]
    Nc = N - args.hot
    return (H * P * args.hot * 4 + H * P * Nc * s + (H * P * 4 if args.cold == "fp8" else 0) + 2 * H * 4
            + args.chunk * (H * P * 2 + H * 4 + G * Nc * 2))


if __name__ == "__main__":
    sys.exit(main())
