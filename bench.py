"""Benchmark of the GDN-stack decode step (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference] [--no-sweep]

Workload (the decode configuration of the reference model's GDN stack): the 30-layer GatedDeltaNet stack of
Qwen3.5-35B-A3B (hidden 2048, Hk 16, Hv 32, dk = dv = 128, conv 4), batched
S=1 decode of B sequences per GPU (default 8).  One step = one decode token for
every sequence through all 30 fused layer steps (gdn_layer_step: conv + SiLU,
q/k norm, gates, gated delta rule on the slot's f32 state, gated RMSNorm).  The
per-layer projection outputs (qkv | z | b | a) are synthetic bf16 resident in
HBM; the in/out projection GEMMs are not part of the timed step.  Pre-existing
states are a seeded random f32 fill (decode cost does not depend on context
length).  A step touches 1.04 GB of state at B=8, far more than the 126 MB L2,
so no L2 flush is needed between steps.

Multi-GPU: one process per GPU (torchrun); each GPU owns its own slot pool of B
sequences (slot-range sharding), there is no collective on the data path; the
NCCL group only provides the barrier and the max-over-ranks time.  value =
all ranks' tokens / max-over-ranks device time ("scaling": "weak").

--impl reference times the CPU restatement of the reference layer (oracle/,
the reference's MLX/Metal path cannot run here) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GDN-stack decode tok/s at B=1..2048 over 1/2/4/8 B200; % HBM roofline"
UNIT = "tok/s"
N_LAYERS = 30
# The layers of a step share its routing tables: layers 2..30 tell the step so (GDN_STEP_TABLES_STABLE), and
# it reads its routing and conv windows while the previous layer's kernel is still running.
STABLE = 1
E2E_REPEATS = 5              # timed e2e runs; the median is reported with the spread
E2E_GROUPS = "1,7,7,7,7,1"   # layers per host<->device copy group in the e2e step (sums to the layer count)
# Algorithmic bytes of one fused decode layer step (per sequence, and per launch constant):
#   state f32 r+w 2*32*128*128*4 + conv bf16 r+w 2*3*8192*2 + qkv 8192*2 + z 4096*2 + a,b 64*2 + out 4096*2
BYTES_PER_SEQ_LAYER = 2 * 32 * 128 * 128 * 4 + 2 * 3 * 8192 * 2 + 8192 * 2 + 4096 * 2 + 64 * 2 + 4096 * 2
#   conv weight 8192*4*2 + A_log 32*4 + dt_bias 32*4 + norm_w 128*2
BYTES_PER_LAUNCH_CONST = 8192 * 4 * 2 + 32 * 4 + 32 * 4 + 128 * 2
assert BYTES_PER_SEQ_LAYER == 4_325_504 and BYTES_PER_LAUNCH_CONST == 66_048
PROJ_LD = 8192 + 4096 + 64     # merged projection output row: qkv | z | b | a


def workload_config(B: int, world: int) -> dict:
    """The `config` of both arms' JSON lines (identical, so the two lines describe the same workload)."""
    return {"workload": f"30-layer GDN stack (hidden 2048, Hk 16, Hv 32), batched S=1 decode, B={B} per GPU",
            "batch_per_gpu": B, "layers": N_LAYERS, "parallelism": f"slot-range shards x{world}",
            "l2": "no flush: state per step %.2f GB > 126 MB L2" % (N_LAYERS * B * BYTES_PER_SEQ_LAYER / 1e9)}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--sweep", default=None, help="comma-separated batch sizes of the sweep (default 1..2048)")
    p.add_argument("--decode-kernel", type=int, default=0,
                   help="gdn_set_decode_kernel mode: 0 by batch size, 1 split, 2 fused, 3 two-kernel")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-mixer", action="store_true")
    p.add_argument("--no-prefill", action="store_true")
    p.add_argument("--no-mixed", action="store_true")
    p.add_argument("--no-sharded", action="store_true")
    p.add_argument("--e2e-groups", default=E2E_GROUPS,
                   help="layers per host<->device copy group of the e2e step, comma separated")
    p.add_argument("--prefill-only", action="store_true",
                   help="run only the chunked-prefill leg and print its result (profiling of that leg)")
    p.add_argument("--prefill-lens", default=None,
                   help="comma-separated prompt lengths for the prefill leg (default: config 4)")
    p.add_argument("--hybrid-only", action="store_true",
                   help="time only the attention and MoE layer bodies of the hybrid decoder (B decode tokens)")
    p.add_argument("--hybrid-ctx", type=int, default=4096, help="cached context of each sequence (hybrid legs)")
    return p.parse_args()


def measured_peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16 tensor-core peak (TFLOP/s) for work timed inside a long step (the prefill leg replays
    seconds of back-to-back layer steps): the sustained figure of MEASURED_PEAKS.json (cuBLAS bf16 looped
    for seconds under the power cap), else its burst figure, else the fallback.  Returns (value, kind)."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured sustained"
        return float(d["bf16_tflops"]), "measured burst"
    return 1400.0, "fallback sustained"


def profiled_traffic():
    """DRAM bytes per launch of the decode layer step from the committed ncu summary, if any."""
    f = ROOT / "profiles" / "gdn_layer_step_decode.txt"
    if not f.exists():
        return None, None
    vals = {}
    for line in f.read_text().splitlines():
        if ":" in line and line.split(":", 1)[0].strip() in ("traffic_bytes_per_seq", "traffic_batch"):
            k, v = line.split(":", 1)
            vals[k.strip()] = float(v.split()[0])
    if "traffic_bytes_per_seq" not in vals:
        return None, None
    return vals["traffic_bytes_per_seq"], vals.get("traffic_batch")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"gdn_bench_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
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
        self.fh.close()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        try:
            self.path.unlink()
        except OSError:
            pass
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ distributed plumbing

def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        return world, rank, local, dist, timedelta
    return 1, 0, 0, None, None


# ------------------------------------------------------------------ CPU baseline (oracle)

def cpu_baseline(batch: int, budget_s: float = 12.0):
    """Time the oracle (CPU restatement of the reference layer) on a bounded sample of the
    same workload: repeated B-sequence decode layer steps; tok/s scaled to the 30-layer stack."""
    import __graft_entry__ as ge
    O = ge.load_oracle()
    synth = ge.load_package().synth
    cfg = synth.GdnConfig(n_layers=1)
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    w = synth.layer_weights(cfg, 0, with_proj=False)
    inp = synth.step_inputs(cfg, batch, seed=0, tag="cpu")
    conv, rec = synth.random_states(cfg, batch, seed=0, tag="cpu")
    cu = np.arange(batch + 1, dtype=np.int32)
    O.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv, rec, cu)   # warm-up
    n = 0
    t0 = time.perf_counter()
    while True:
        _, conv, rec, _ = O.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv, rec, cu)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    per_stack_step = dt / n * N_LAYERS
    return {"value": batch / per_stack_step, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} oracle decode layer steps of B={batch} in {dt:.1f} s, scaled x{N_LAYERS} layers/step"}


def run_reference(args):
    world, rank, local, dist, _ = dist_setup(args.gpus)
    if rank != 0:
        return
    import __graft_entry__ as ge
    O = ge.load_oracle()
    synth = ge.load_package().synth
    cfg = synth.GdnConfig(n_layers=1)
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    B = args.batch
    # Bounded sample per step: L_S of the 30 layers, scaled to the full stack.
    L_S = 3
    ws = [synth.layer_weights(cfg, l, with_proj=False) for l in range(L_S)]
    inps = [synth.step_inputs(cfg, B, seed=0, tag=f"ref{l}") for l in range(L_S)]
    states = [synth.random_states(cfg, B, seed=0, tag=f"ref{l}") for l in range(L_S)]
    cu = np.arange(B + 1, dtype=np.int32)

    def step():
        for l in range(L_S):
            conv, rec = states[l]
            _, conv, rec, _ = O.layer_step(cfg, ws[l], inps[l]["qkv"], inps[l]["z"], inps[l]["ab"], conv, rec, cu)
            states[l] = (conv, rec)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    ms_per_step = dt / args.steps * 1e3 * N_LAYERS / L_S
    value = B / (ms_per_step / 1e3)
    sample = f"{L_S} of {N_LAYERS} layers per step (scaled x{N_LAYERS // L_S}), B={B} decode, {args.steps} steps"
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 state, bf16 io", "data": "synthetic",
            "config": workload_config(B, args.gpus),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample + "; rank 0 times one shard's B on the host cores; CPU restatement "
                                                "of the reference layer (MLX/Metal unavailable)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm

def _cudart():
    """The CUDA runtime torch already loaded (used only to fill the pool with random state)."""
    for line in open("/proc/self/maps"):
        if "libcudart.so" in line:
            return C.CDLL(line.split()[-1])
    raise RuntimeError("libcudart not loaded")


def bind_to_gpu_numa_node(torch, dev):
    """Restrict this process to the host cores of its GPU's NUMA node, so pinned host buffers allocated
    afterwards (first touch) sit next to the GPU's PCIe root and the host<->device copies do not cross
    the inter-socket link.  Affects this process only.  Returns a description, or None when the node is
    unknown."""
    try:
        p = torch.cuda.get_device_properties(dev)
        bdf = "%04x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
        node = int(Path(f"/sys/bus/pci/devices/{bdf}/numa_node").read_text().strip())
        if node < 0:
            return None
        cpus = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return {"node": node, "cpus": len(cpus), "pci": bdf}
    except (OSError, ValueError, AttributeError):
        return None


def _gpu_uuid(torch, dev):
    """nvidia-smi -i identifier of this process's GPU (UUID; the CUDA index may be remapped)."""
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev.index)


# Bytes of one mixer layer's projection weights: in_proj (8192 + 4096 + 64 rows) and out_proj, bf16.
MIXER_WEIGHT_BYTES = ((8192 + 4096 + 64) * 2048 + 2048 * 4096) * 2
assert MIXER_WEIGHT_BYTES == 67_371_008


def _time_stack(torch, lib, abi, pool, arr, h, slots, cu, B, cfg, stream, barrier, dist, args):
    """Device ms and e2e ms (x in from pinned host, h out) of `args.steps` graph-replayed stack steps."""
    sp = C.c_void_p(stream.cuda_stream)

    def step():
        rc = lib.gdn_stack_step(pool.h, arr, C.c_void_p(h.data_ptr()), cfg.hidden, C.c_void_p(slots.data_ptr()),
                                C.c_void_p(cu.data_ptr()), B, B, sp)
        if rc:
            abi.check(rc, "gdn_stack_step")

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            g.replay()
    stream.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            g.replay()
        e1.record(stream)
    e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    # e2e: this step's hidden states in (pinned host -> device), the updated hidden states out
    x_host = torch.empty((B, cfg.hidden), dtype=torch.bfloat16).pin_memory()
    x_host.copy_(h.cpu())
    y_host = torch.empty_like(x_host).pin_memory()
    with torch.cuda.stream(stream):
        for _ in range(3):
            h.copy_(x_host, non_blocking=True)
            g.replay()
            y_host.copy_(h, non_blocking=True)
    stream.synchronize()
    barrier()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            h.copy_(x_host, non_blocking=True)
            g.replay()
            y_host.copy_(h, non_blocking=True)
        e1.record(stream)
    e1.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms, e2e_ms], device=h.device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0].item()), float(t[1].item())
    del g
    return ms, e2e_ms, x_host.numel() * 2, y_host.numel() * 2


# 4-bit (MLX affine, group 64) bytes of one layer's projections: codes + bf16 scale and bias per group.
MIXER_WEIGHT_BYTES_Q4 = ((8192 + 4096 + 64) * 2048 + 2048 * 4096) // 2 + \
    ((8192 + 4096 + 64) * 2048 + 2048 * 4096) // 64 * 4
assert MIXER_WEIGHT_BYTES_Q4 == 18_948_096


def run_mixer_stack(torch, dev, gen, cfg, gdn, abi, lib, pool, B, stream, barrier, dist, world, args, hbm_peak):
    """Config 2 through gdn_stack_step: h <- h + mixer_l(rms_norm(h)) over 30 layers, twice: with bf16
    projections (cuBLASLt) and with MLX 4-bit projections (the reference's quantized checkpoint format;
    the weight-streaming tcgen05 kernel, weights dequantized on chip).  Device tok/s, and e2e with the
    step's x copied in and h copied out."""
    import importlib
    synth = importlib.import_module("qwen_mlx_b200.synth")
    plain, q4, tiled = [], [], []
    keep = []
    n_in = 8192 + 4096 + 64
    for l in range(N_LAYERS):
        w = synth.layer_weights(cfg, l, with_proj=False)
        step = gdn.LayerWeights(w, dev)
        w_in = (torch.randn((n_in, cfg.hidden), device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        w_out = (torch.randn((cfg.hidden, cfg.z_dim), device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        pre = torch.ones(cfg.hidden, dtype=torch.bfloat16, device=dev)
        # synthetic 4-bit weights: random codes, scales U(0, 0.005), biases N(0, 0.005^2) (timing only)
        qt = []
        for rows, cols in ((n_in, cfg.hidden), (cfg.hidden, cfg.z_dim)):
            wq = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows, cols // 8), dtype=torch.int32, device=dev, generator=gen)
            sc = (torch.rand((rows, cols // 64), device=dev, generator=gen) * 0.005).to(torch.bfloat16)
            bi = (torch.randn((rows, cols // 64), device=dev, generator=gen) * 0.005).to(torch.bfloat16)
            qt.append(gdn.tile_weight_q4(wq, sc, bi))
        bt = (gdn.tile_weight(w_in), gdn.tile_weight(w_out))   # bf16 tiles: the repo's streaming kernels
        keep.append((step, w_in, w_out, pre, qt, bt))
        plain.append(abi.GdnMixerWeightsC(step.c, w_in.data_ptr(), w_out.data_ptr(), pre.data_ptr(),
                                          None, None, None, None))
        tiled.append(abi.GdnMixerWeightsC(step.c, w_in.data_ptr(), w_out.data_ptr(), pre.data_ptr(),
                                          bt[0].data_ptr(), bt[1].data_ptr(), None, None))
        q4.append(abi.GdnMixerWeightsC(step.c, None, None, pre.data_ptr(), None, None, qt[0].data_ptr(),
                                       qt[1].data_ptr()))
    arr_p = (abi.GdnMixerWeightsC * N_LAYERS)(*plain)
    arr_q = (abi.GdnMixerWeightsC * N_LAYERS)(*q4)
    arr_t = (abi.GdnMixerWeightsC * N_LAYERS)(*tiled)
    h = torch.randn((B, cfg.hidden), device=dev, generator=gen).to(torch.bfloat16)
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
    ms, e2e_ms, hb, db = _time_stack(torch, lib, abi, pool, arr_p, h, slots, cu, B, cfg, stream, barrier, dist, args)
    ms_q, e2e_q, _, _ = _time_stack(torch, lib, abi, pool, arr_q, h, slots, cu, B, cfg, stream, barrier, dist, args)
    ms_t, e2e_t, _, _ = _time_stack(torch, lib, abi, pool, arr_t, h, slots, cu, B, cfg, stream, barrier, dist, args)
    step_bytes = N_LAYERS * (MIXER_WEIGHT_BYTES + B * BYTES_PER_SEQ_LAYER + BYTES_PER_LAUNCH_CONST)
    step_bytes_q = N_LAYERS * (MIXER_WEIGHT_BYTES_Q4 + B * BYTES_PER_SEQ_LAYER + BYTES_PER_LAUNCH_CONST)
    return {"tok_s": world * B * args.steps / (ms / 1e3), "ms_per_step": ms / args.steps,
            "hbm_frac_of_measured": step_bytes / (ms / args.steps / 1e3) / 1e9 / hbm_peak,
            "bytes_per_step": step_bytes,
            "e2e_tok_s": world * B * args.steps / (e2e_ms / 1e3), "h2d_bytes_per_step": hb,
            "d2h_bytes_per_step": db,
            "note": "30 x (pre-norm + in_proj GEMM + gdn_layer_step + out_proj GEMM + residual); bf16 GEMMs "
                    "are cuBLASLt",
            "q4": {"tok_s": world * B * args.steps / (ms_q / 1e3), "ms_per_step": ms_q / args.steps,
                   "hbm_frac_of_measured": step_bytes_q / (ms_q / args.steps / 1e3) / 1e9 / hbm_peak,
                   "bytes_per_step": step_bytes_q, "e2e_tok_s": world * B * args.steps / (e2e_q / 1e3),
                   "note": "same stack, MLX 4-bit (group 64) projections on the weight-streaming tcgen05 "
                           "kernel; synthetic random codes"},
            "bf16_tiles": {"tok_s": world * B * args.steps / (ms_t / 1e3), "ms_per_step": ms_t / args.steps,
                           "hbm_frac_of_measured": step_bytes / (ms_t / args.steps / 1e3) / 1e9 / hbm_peak,
                           "bytes_per_step": step_bytes, "e2e_tok_s": world * B * args.steps / (e2e_t / 1e3),
                           "note": "same stack, bf16 projections from the tiled weight copies on this repo's "
                                   "streaming tcgen05 kernels (<= 16 tokens: weight stages in shared memory)"}}


# Prefill (chunked WY) algorithmic flops per token per layer, chunk 64: 6*dk*dv + 2*C*(3*dk + 2*dv) per
# v-head (state readout, state update, W S0^T, and the intra-chunk K K^T, Q K^T, T V, T K, P D), x 32 heads.
WY_FLOPS_PER_TOKEN_LAYER = 32 * (6 * 128 * 128 + 2 * 64 * (3 * 128 + 2 * 128))
assert WY_FLOPS_PER_TOKEN_LAYER == 5_767_168
CONFIG4_LENS = [512, 1024, 2048, 3000, 4096, 5000, 6144, 8192]
TOKEN_IO_BYTES = 8192 * 2 + 4096 * 2 + 64 * 2 + 4096 * 2    # qkv, z, a/b in; gated output out (per token, layer)
STATE_BYTES_PER_SEQ_LAYER = BYTES_PER_SEQ_LAYER - TOKEN_IO_BYTES


def _time_ragged(torch, dev, cfg, abi, lib, lws, stream, barrier, dist, mpool, plans, warm, n_tab, per_layer_io,
                 gen):
    """Run `plans` (per step: pool slot ids, cu_seqlens) as one packed gdn_layer_step_ex call per layer.  Each
    step is one CUDA graph (token counts change every step, so every plan has its own graph, captured before
    the timed region): the host->device copy of the step's routing tables from its own pinned host buffer,
    then the 30 layer calls.  The first `warm` steps are untimed.  Returns (device ms of the timed steps, max
    over ranks, timed plans, this rank's own ms).  With `per_layer_io` every layer reads its own projection
    rows; otherwise all layers share one input and one output buffer (larger than L2 at these token counts)."""
    n_max = max(int(c[-1]) for _, c in plans)
    mpool.reserve_tokens(n_max)
    n_io = N_LAYERS if per_layer_io else 1
    proj = torch.randn((n_io, n_max, PROJ_LD), device=dev, generator=gen).to(torch.bfloat16)
    out = torch.empty((n_io, n_max, cfg.z_dim), dtype=torch.bfloat16, device=dev)
    sp = C.c_void_p(stream.cuda_stream)
    ios = [abi.GdnStepIOC(proj[i].data_ptr(), PROJ_LD, proj[i].data_ptr() + 8192 * 2, PROJ_LD,
                          proj[i].data_ptr() + (8192 + 4096) * 2, PROJ_LD, out[i].data_ptr(), cfg.z_dim)
           for i in range(n_io)]
    tabs_h, tabs_d = [], []
    for sl, cu in plans:
        t = torch.zeros(2 * (n_tab + 1), dtype=torch.int32).pin_memory()
        t[:len(sl)] = torch.from_numpy(sl)
        t[n_tab + 1:n_tab + 2 + len(sl)] = torch.from_numpy(cu)
        tabs_h.append(t)
        tabs_d.append(torch.empty(2 * (n_tab + 1), dtype=torch.int32, device=dev))

    def step(k):
        sl, cu = plans[k]
        n = len(sl)
        tab_d = tabs_d[k]
        tab_d.copy_(tabs_h[k], non_blocking=True)
        for l in range(N_LAYERS):
            rc = lib.gdn_layer_step_ex(mpool.h, l, C.byref(lws[l].c), C.byref(ios[l % n_io]),
                                       C.c_void_p(tab_d.data_ptr()), C.c_void_p(tab_d.data_ptr() + (n_tab + 1) * 4),
                                       n, int(cu[-1]), STABLE if l else 0, sp)
            if rc:
                abi.check(rc, "gdn_layer_step_ex")

    with torch.cuda.stream(stream):
        step(0)                         # eager run: kernel attributes are set outside any capture
    stream.synchronize()
    graphs = []
    for k in range(len(plans)):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(k)
        graphs.append(g)
    with torch.cuda.stream(stream):
        for k in range(warm):
            graphs[k].replay()
    stream.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for k in range(warm, len(plans)):
            graphs[k].replay()
        e1.record(stream)
    e1.synchronize()
    barrier()
    own_ms = ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    assert mpool.check() == 0
    del graphs, proj, out
    return ms, plans[warm:], own_ms


def _per_rank(torch, dev, dist, world, own_ms, timed):
    """Per-rank breakdown of a ragged leg (gathered to every rank): device ms of the timed steps, tokens,
    prefill chunks and the longest chunk -- the rank with the longest chunk chain sets the max-over-ranks
    time."""
    tokens = sum(int(c[-1]) for _, c in timed)
    lens = np.concatenate([np.diff(c) for _, c in timed])
    chunks = lens[lens > 1]
    mine = [own_ms, tokens, len(chunks), int(chunks.max()) if len(chunks) else 0,
            int(sum(-(-int(x) // 64) for x in chunks))]
    t = torch.tensor(mine, device=dev, dtype=torch.float64)
    if dist is not None:
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        rows = [o.tolist() for o in out]
    else:
        rows = [t.tolist()]
    return [{"rank": r, "ms": round(row[0], 3), "tokens": int(row[1]), "prefill_chunks": int(row[2]),
             "longest_chunk": int(row[3]), "wy_chunks_of_64": int(row[4])} for r, row in enumerate(rows)]


def _ragged_summary(ms, timed, world, hbm_peak):
    tokens = sum(int(c[-1]) for _, c in timed)
    seqs = sum(len(sl) for sl, _ in timed)
    step_bytes = sum(N_LAYERS * (len(sl) * STATE_BYTES_PER_SEQ_LAYER + int(c[-1]) * TOKEN_IO_BYTES
                                 + BYTES_PER_LAUNCH_CONST) for sl, c in timed)
    return {"steps": len(timed), "tokens_per_gpu": tokens, "sequence_steps_per_gpu": seqs,
            "tok_s": world * tokens / (ms / 1e3), "ms_per_step": ms / len(timed),
            "hbm_frac_of_measured": step_bytes / (ms / 1e3) / 1e9 / hbm_peak}


def run_mixed(torch, dev, gen, cfg, gdn, abi, lib, lws, stream, barrier, dist, world, args, hbm_peak):
    """Config 3 (ragged continuous batching): a 256-slot pool with 64 live sequences holding prior state;
    every step a seeded 50-100% subset is active and ~10% of the active ones carry a prefill chunk of
    U[1, 512] tokens, all packed in one call per layer (30 fused layer steps).  Token counts change every
    step, so every step is its own CUDA graph; each graph uploads its step's tables first."""
    rng = np.random.default_rng(1234)
    n_slots, n_live, n_steps, warm = 256, 64, 12, 3
    slots_live = rng.permutation(n_slots)[:n_live].astype(np.int32)
    plans = []
    for _ in range(n_steps):
        n_act = int(rng.integers(n_live // 2, n_live + 1))
        act = rng.permutation(n_live)[:n_act]
        n_pref = max(1, int(round(0.1 * n_act)))
        lens = np.ones(n_act, np.int64)
        lens[:n_pref] = rng.integers(1, 513, n_pref)
        order = rng.permutation(n_act)
        act, lens = act[order], lens[order]
        plans.append((slots_live[act], np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)))
    mpool = gdn.StatePool(cfg, n_slots=n_slots, device=dev.index)
    ms, timed, _ = _time_ragged(torch, dev, cfg, abi, lib, lws, stream, barrier, dist, mpool, plans, warm, n_live,
                                True, gen)
    mpool.close()
    return {"workload": "config3: 256-slot pool, 64 live, 50-100% active per step, ~10% of them with a prefill "
                        "chunk U[1,512], 30 fused layer steps, one CUDA graph per step (table upload inside)",
            **_ragged_summary(ms, timed, world, hbm_peak)}


def config5_plans(rank: int, n_steps: int, slots_per_gpu: int = 256):
    """Step plans of config 5 for the GPU owning global slots [256 rank, 256 (rank + 1)): all 256 local
    sequences step every time; a seeded 10% of them carry a prefill chunk of U[64, 1024] tokens and the rest
    one decode token, packed in a random order.  Context lengths are drawn log-uniform in [16, 32768] as the
    workload states; they decide nothing in a GDN step, whose state per sequence has a fixed size, so the
    pre-existing state is a seeded random fill."""
    rng = np.random.default_rng(5000 + rank)
    ctx = np.exp(rng.uniform(np.log(16), np.log(32768), slots_per_gpu)).astype(np.int64)
    plans = []
    for _ in range(n_steps):
        n_pref = int(round(0.1 * slots_per_gpu))
        lens = np.ones(slots_per_gpu, np.int64)
        lens[:n_pref] = rng.integers(64, 1025, n_pref)
        order = rng.permutation(slots_per_gpu)
        plans.append((order.astype(np.int32), np.concatenate([[0], np.cumsum(lens[order])]).astype(np.int32)))
    return plans, ctx


def run_sharded(torch, dev, gen, cfg, gdn, abi, lib, pool, lws, stream, barrier, dist, world, rank, args,
                hbm_peak):
    """Config 5 (sharded serving, weak scaling): each GPU owns 256 slots of the 256 * world sequences (2048 at
    8 GPUs), partitioned by slot range, and runs its own packed steps with no exchange between GPUs.  Time is
    the max over ranks; tok/s is the whole job's."""
    n_steps, warm = 11, 3
    plans, ctx = config5_plans(rank, n_steps)
    own = pool is None or pool.n_slots < 256
    mpool = gdn.StatePool(cfg, n_slots=256, device=dev.index) if own else pool
    ms, timed, own_ms = _time_ragged(torch, dev, cfg, abi, lib, lws, stream, barrier, dist, mpool, plans, warm,
                                     256, False, gen)
    ranks = _per_rank(torch, dev, dist, world, own_ms, timed)
    if own:
        mpool.close()
    return {"workload": "config5: 256 slots per GPU (slot-range shards, %d sequences in all), every step 90%% "
                        "S=1 decode + 10%% prefill chunks U[64,1024], context log-U[16,32768], 30 fused layer "
                        "steps, one CUDA graph per step (table upload inside), no collective" % (256 * world),
            "median_context_rank0": int(np.median(ctx)), **_ragged_summary(ms, timed, world, hbm_peak),
            "per_rank": ranks}


def run_prefill(torch, dev, gen, cfg, gdn, abi, lib, pool, lws, stream, barrier, dist, world, args, tc_peak):
    """Config 4: 8 prompts packed in one call per layer, zero initial state, 30 layers (fused steps).
    Segments of >= 32 tokens run the tcgen05 chunked kernel."""
    lens = [int(x) for x in args.prefill_lens.split(",")] if args.prefill_lens else CONFIG4_LENS
    cu_h = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    N = int(cu_h[-1])
    pool.reserve_tokens(N)
    proj = torch.randn((N, PROJ_LD), device=dev, generator=gen).to(torch.bfloat16)
    out = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=dev)
    slots = torch.arange(len(lens), dtype=torch.int32, device=dev)
    cu = torch.from_numpy(cu_h).to(dev)
    io = abi.GdnStepIOC(proj.data_ptr(), PROJ_LD, proj.data_ptr() + 8192 * 2, PROJ_LD,
                        proj.data_ptr() + (8192 + 4096) * 2, PROJ_LD, out.data_ptr(), cfg.z_dim)
    slots_h = np.arange(len(lens), dtype=np.int32)
    sp = C.c_void_p(stream.cuda_stream)

    def step():
        pool.reset(slots_h, stream)                     # prompts start from a zero state
        for l in range(N_LAYERS):
            rc = lib.gdn_layer_step_ex(pool.h, l, C.byref(lws[l].c), C.byref(io), C.c_void_p(slots.data_ptr()),
                                       C.c_void_p(cu.data_ptr()), len(lens), N, STABLE if l else 0, sp)
            if rc:
                abi.check(rc, "gdn_layer_step_ex")

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    steps = max(2, min(args.steps, 5))
    with torch.cuda.stream(stream):
        g.replay()
    stream.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            g.replay()
        e1.record(stream)
    e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del g
    ms_step = ms / steps
    flops = N * N_LAYERS * WY_FLOPS_PER_TOKEN_LAYER
    name = "config4" if lens == CONFIG4_LENS else "custom"
    peak, peak_kind = tc_peak
    return {"workload": "%s: prompts %s packed in one call, zero state, 30 fused layer steps" % (name, lens),
            "tokens": N, "tok_s": world * N / (ms_step / 1e3), "ms_per_step": ms_step,
            "algorithmic_tflops": flops / (ms_step / 1e3) / 1e12, "tensor_peak_tflops": peak,
            "tensor_peak_kind": peak_kind,
            "tensor_frac_of_measured": flops / (ms_step / 1e3) / 1e12 / peak,
            "flops_per_token_layer": WY_FLOPS_PER_TOKEN_LAYER}


def run_hybrid(args):
    """Decode-step timing of the hybrid decoder's other layers at Qwen3.5-35B-A3B shapes, through the public API
    (eager calls; the attention call uploads its routing table each call): one attention layer body (16 q / 2 kv
    heads of 256, every sequence `--hybrid-ctx` keys deep) and one MoE block (256 4-bit experts, top-8, shared
    expert).  Roofline: the attention reads every cached key and value once per kv head; the MoE reads the
    routed experts' 4-bit weights (codes, scales and biases) once, the shared expert's and the router's."""
    import torch
    import __graft_entry__ as ge
    ge.load_package()
    import importlib
    synth = importlib.import_module("qwen_mlx_b200.synth")
    gdn = importlib.import_module("qwen_mlx_b200.gdn")
    hy = importlib.import_module("qwen_mlx_b200.hybrid")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, ctx = args.batch, args.hybrid_ctx
    hbm_peak, peak_kind = measured_peaks()
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    steps = max(args.steps, 20)

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / steps * 1e3   # us per call

    acfg = hy.AttnConfig(max_ctx=ctx)
    cache = hy.KVCache(acfg, B, dev)
    cache.k.normal_(generator=gen)
    cache.v.normal_(generator=gen)
    D = acfg.n_heads * acfg.head_dim
    qf = torch.randn((B, 2 * D), device=dev, generator=gen).to(torch.bfloat16)
    kin = torch.randn((B, acfg.n_kv_heads * acfg.head_dim), device=dev, generator=gen).to(torch.bfloat16)
    vin = torch.randn_like(kin)
    gain = torch.ones(acfg.head_dim, device=dev, dtype=torch.bfloat16)
    slots, cu, pos = list(range(B)), list(range(B + 1)), [ctx - 1] * B
    ws = torch.empty(hy.attn_workspace_bytes(acfg, B, ctx), dtype=torch.uint8, device=dev)
    out = torch.empty((B, D), dtype=torch.bfloat16, device=dev)
    us_attn = timed(lambda: hy.attn_step(cache, qf, kin, vin, gain, gain, slots, cu, pos, out=out, workspace=ws))
    attn_bytes = B * acfg.n_kv_heads * ctx * acfg.head_dim * 2 * 2

    mcfg = hy.MoeConfig()
    mw_np = synth.moe_weights(mcfg.hidden, mcfg.n_experts, mcfg.moe_inter, mcfg.shared_inter, seed=3)
    mw = hy.MoeWeights(mw_np, dev)
    x = torch.randn((B, mcfg.hidden), device=dev, generator=gen).to(torch.bfloat16)
    mws = torch.empty(hy.moe_workspace_bytes(mcfg, B), dtype=torch.uint8, device=dev)
    mout = torch.empty((B, mcfg.hidden), dtype=torch.bfloat16, device=dev)
    us_moe = timed(lambda: hy.moe_step(mcfg, mw, x, out=mout, workspace=mws))
    ids, _, _ = hy.moe_route(mcfg, mw, x)
    n_exp = int(torch.unique(ids).numel())

    def q4_bytes(rows, cols):
        return rows * cols // 2 + 2 * 2 * rows * (cols // 64)

    per_expert = 2 * q4_bytes(mcfg.moe_inter, mcfg.hidden) + q4_bytes(mcfg.hidden, mcfg.moe_inter)
    shared = 2 * q4_bytes(mcfg.shared_inter, mcfg.hidden) + q4_bytes(mcfg.hidden, mcfg.shared_inter)
    moe_bytes = n_exp * per_expert + shared + mcfg.n_experts * mcfg.hidden * 2
    res = {
        "workload": f"hybrid layers, batched S=1 decode, B={B}, {ctx} cached keys per sequence",
        "attention": {"us_per_layer": us_attn, "alg_bytes": attn_bytes,
                      "achieved_gbs": attn_bytes / us_attn / 1e3, "hbm_frac": attn_bytes / us_attn / 1e3 / hbm_peak,
                      "config": "16 q heads, 2 kv heads, head_dim 256, rotary 64; gdn_attn_step eager"},
        "moe": {"us_per_layer": us_moe, "experts_touched": n_exp, "alg_bytes": moe_bytes,
                "achieved_gbs": moe_bytes / us_moe / 1e3, "hbm_frac": moe_bytes / us_moe / 1e3 / hbm_peak,
                "config": "256 experts (4-bit, group 64), top-8, moe/shared intermediate 512; gdn_moe_step eager"},
        "hbm_peak_gbs": hbm_peak, "peak_kind": peak_kind,
    }
    print(json.dumps({"hybrid": res}), flush=True)


def run_ours(args):
    import torch
    world, rank, local, dist, timedelta = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if dist is not None:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=dev)
    import __graft_entry__ as ge
    pkg = ge.load_package()
    import importlib
    synth = importlib.import_module("qwen_mlx_b200.synth")
    gdn = importlib.import_module("qwen_mlx_b200.gdn")
    abi = importlib.import_module("qwen_mlx_b200.abi")
    lib = abi.lib()

    cfg = synth.GdnConfig(n_layers=N_LAYERS)
    B = args.batch
    sweep_bs = [] if (args.no_sweep or world > 1 or args.prefill_only) else (
        [int(x) for x in args.sweep.split(",")] if args.sweep else [1, 2, 4, 8, 16, 32, 64, 256, 1024, 2048])
    abi.check(lib.gdn_set_decode_kernel(args.decode_kernel), "gdn_set_decode_kernel")
    n_slots = max([B] + sweep_bs)
    if args.prefill_only:
        n_slots = max(n_slots, len(args.prefill_lens.split(",")) if args.prefill_lens else len(CONFIG4_LENS))
    pool = gdn.StatePool(cfg, n_slots=n_slots, device=local)
    cudart = _cudart()
    cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    tile = cfg.hv * cfg.dv * cfg.dk
    fill = (torch.randn(n_slots * tile, device=dev, generator=gen) * 0.05).float()
    cfill = torch.randn(n_slots * 3 * cfg.conv_dim, device=dev, generator=gen).to(torch.bfloat16)
    for l in range(N_LAYERS):
        rec_p, conv_p = pool.layer_state_ptrs(l)
        assert cudart.cudaMemcpy(rec_p, fill.data_ptr(), fill.numel() * 4, 3) == 0
        assert cudart.cudaMemcpy(conv_p, cfill.data_ptr(), cfill.numel() * 2, 3) == 0
    del fill, cfill

    # weights (synthetic, seeded) and per-layer projection outputs resident in HBM
    lws = [gdn.LayerWeights(synth.layer_weights(cfg, l, with_proj=False), dev) for l in range(N_LAYERS)]
    slots_all = torch.arange(n_slots, dtype=torch.int32, device=dev)
    cu_all = torch.arange(n_slots + 1, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    sp = C.c_void_p(stream.cuda_stream)

    def buffers(b):
        """Contiguous per-layer projection outputs [L, b, qkv|z|b|a] and step outputs [L, b, Hv*dv]."""
        proj = torch.randn((N_LAYERS, b, PROJ_LD), device=dev, generator=gen).to(torch.bfloat16)
        out = torch.empty((N_LAYERS, b, cfg.z_dim), dtype=torch.bfloat16, device=dev)
        return proj, out

    def make_io(proj, out, l):
        base = proj[l]
        return abi.GdnStepIOC(base.data_ptr(), PROJ_LD, base.data_ptr() + 8192 * 2, PROJ_LD,
                              base.data_ptr() + (8192 + 4096) * 2, PROJ_LD, out[l].data_ptr(), cfg.z_dim)

    def step_fn(b, proj, out):
        ios = [make_io(proj, out, l) for l in range(N_LAYERS)]
        wcs = [lw.c for lw in lws]
        sptr = C.c_void_p(slots_all.data_ptr())
        cptr = C.c_void_p(cu_all.data_ptr())

        def step():
            for l in range(N_LAYERS):
                rc = lib.gdn_layer_step_ex(pool.h, l, C.byref(wcs[l]), C.byref(ios[l]), sptr, cptr, b, b,
                                           STABLE if l else 0, sp)
                if rc:
                    abi.check(rc, "gdn_layer_step_ex")
        return step

    def capture(b, proj, out):
        step = step_fn(b, proj, out)
        with torch.cuda.stream(stream):
            step()                      # eager warm-up (also validates arguments)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        return g

    def barrier():
        if dist is not None:
            dist.barrier()

    def time_graph(g, steps, warmup):
        """Device time of `steps` replays of the step graph; replays run on `stream`, events on `stream`."""
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                g.replay()
        stream.synchronize()
        barrier()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                g.replay()
            e1.record(stream)
        e1.synchronize()
        torch.cuda.synchronize(dev)
        barrier()
        return e0.elapsed_time(e1)

    def soak(g, seconds):
        """Replay the step graph for `seconds` (clock sampling under the same load)."""
        t_end = time.perf_counter() + seconds
        with torch.cuda.stream(stream):
            while time.perf_counter() < t_end:
                for _ in range(20):
                    g.replay()
                stream.synchronize()

    hbm_peak, peak_kind = measured_peaks()
    all_cpus = os.sched_getaffinity(0)
    numa = bind_to_gpu_numa_node(torch, dev)

    if args.prefill_only:
        res = run_prefill(torch, dev, gen, cfg, gdn, abi, lib, pool, lws, stream, barrier, dist, world, args,
                          measured_tensor_peak())
        if rank == 0:
            print(json.dumps({"prefill": res}), flush=True)
        pool.close()
        if dist is not None:
            dist.destroy_process_group()
        return

    # ---- headline: B sequences per GPU
    proj_h, out_h = buffers(B)
    g = capture(B, proj_h, out_h)
    clocks = ClockSampler(_gpu_uuid(torch, dev))
    clocks.start()
    soak(g, 1.0)
    ms = time_graph(g, args.steps, max(args.warmup, 3))
    soak(g, 0.5)
    clk = clocks.stop()
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = world * B * args.steps / (ms / 1e3)
    gpu_launches = args.steps * N_LAYERS * 2     # gdn_prep_kernel + gdn_recur_kernel per layer

    # ---- roofline of the dominant kernel (the fused layer step), per launch
    launch_ms = ms_per_step / N_LAYERS     # average launch duration inside the timed graph (gaps included)
    alg_bytes = B * BYTES_PER_SEQ_LAYER + BYTES_PER_LAUNCH_CONST
    achieved = alg_bytes / (launch_ms / 1e3) / 1e9
    tr_per_seq, _ = profiled_traffic()
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                "traffic": (tr_per_seq * B if tr_per_seq else None), "peak_kind": peak_kind,
                "traffic_source": "profiles/gdn_layer_step_decode.txt: per-sequence DRAM reads + the bytes the SMs "
                                  "write into L2 (all of which reach DRAM) of one K1 + K2 pair at B=63, x B",
                "kernel": "gdn_layer_step = gdn_prep_kernel + gdn_recur_kernel (PDL-chained)",
                "launch_us": launch_ms * 1e3,
                "alg_bytes_per_launch": alg_bytes,
                "step_frac": (B * N_LAYERS * BYTES_PER_SEQ_LAYER + N_LAYERS * BYTES_PER_LAUNCH_CONST)
                / (ms_per_step / 1e3) / 1e9 / hbm_peak}

    # ---- e2e through the public API with host buffers (pinned), copies inside the timed region.
    # Every step copies each layer's projection outputs in and each layer's output back.  The copies run on
    # two copy streams in groups of layers (--e2e-groups): group g's input copy gates group g's steps and its
    # output copy follows them, so the host link overlaps the compute (one CUDA graph per step).  A one-layer
    # first group lets the compute start after one layer's input; a one-layer last group leaves one layer's
    # output to drain; the groups in between are large because each copy has a fixed cost of a few us and each
    # cross-stream edge interrupts the programmatic launch overlap of consecutive steps.
    in_host = torch.empty((N_LAYERS, B, PROJ_LD), dtype=torch.bfloat16).pin_memory()
    in_host.copy_(proj_h.cpu())
    out_host = torch.empty((N_LAYERS, B, cfg.z_dim), dtype=torch.bfloat16).pin_memory()
    h2d = torch.cuda.Stream(device=dev)
    d2h = torch.cuda.Stream(device=dev)
    ios_e = [make_io(proj_h, out_h, l) for l in range(N_LAYERS)]
    wcs_e = [lw.c for lw in lws]
    sizes = [int(v) for v in args.e2e_groups.split(",")]
    if sum(sizes) != N_LAYERS or min(sizes) < 1:
        raise SystemExit(f"--e2e-groups must be positive sizes summing to {N_LAYERS}")
    starts = np.cumsum([0] + sizes)
    groups = [(int(starts[i]), int(starts[i + 1])) for i in range(len(sizes))]

    def e2e_body():
        ev_in = [torch.cuda.Event() for _ in groups]
        ev_out = [torch.cuda.Event() for _ in groups]
        h2d.wait_stream(stream)
        d2h.wait_stream(stream)
        with torch.cuda.stream(h2d):
            for gi, (a, b) in enumerate(groups):
                proj_h[a:b].copy_(in_host[a:b], non_blocking=True)
                ev_in[gi].record(h2d)
        for gi, (a, b) in enumerate(groups):
            stream.wait_event(ev_in[gi])
            for l in range(a, b):
                rc = lib.gdn_layer_step_ex(pool.h, l, C.byref(wcs_e[l]), C.byref(ios_e[l]),
                                           C.c_void_p(slots_all.data_ptr()), C.c_void_p(cu_all.data_ptr()), B, B,
                                           STABLE if l else 0, sp)
                if rc:
                    abi.check(rc, "gdn_layer_step_ex")
            ev_out[gi].record(stream)
            d2h.wait_event(ev_out[gi])
            with torch.cuda.stream(d2h):
                out_host[a:b].copy_(out_h[a:b], non_blocking=True)
        stream.wait_stream(h2d)
        stream.wait_stream(d2h)

    with torch.cuda.stream(stream):
        e2e_body()                      # eager run (validates the stream wiring)
    stream.synchronize()
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e, stream=stream):
        e2e_body()

    def e2e_step():
        with torch.cuda.stream(stream):
            g_e2e.replay()

    for _ in range(max(args.warmup, 3)):
        e2e_step()
    stream.synchronize()
    # E2E_REPEATS timed runs of K steps each (max over ranks per run); the reported value is their median
    e2e_runs = []
    for _ in range(E2E_REPEATS):
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        e1.synchronize()
        barrier()
        e2e_ms = e0.elapsed_time(e1)
        if dist is not None:
            t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e_runs.append(world * B * args.steps / (e2e_ms / 1e3))
    del g_e2e
    e2e = {"value": statistics.median(e2e_runs), "unit": UNIT,
           "h2d_bytes_per_step": in_host.numel() * 2, "d2h_bytes_per_step": out_host.numel() * 2,
           "repeats": [round(v, 1) for v in e2e_runs], "min": min(e2e_runs), "max": max(e2e_runs),
           "host_numa": numa}

    # ---- config-4 prefill on the chunked tensor-core path
    prefill = None
    if not args.no_prefill:
        prefill = run_prefill(torch, dev, gen, cfg, gdn, abi, lib, pool, lws, stream, barrier, dist, world, args,
                              measured_tensor_peak())

    # ---- config-3 continuous batching (ragged prefill chunks mixed with decode)
    mixed = None
    if not args.no_mixed:
        mixed = run_mixed(torch, dev, gen, cfg, gdn, abi, lib, lws, stream, barrier, dist, world, args, hbm_peak)

    # ---- config-5 sharded serving: 256 slots per GPU, 90% decode / 10% prefill chunks, no collective
    sharded = None
    if not args.no_sharded:
        sharded = run_sharded(torch, dev, gen, cfg, gdn, abi, lib, pool, lws, stream, barrier, dist, world, rank,
                              args, hbm_peak)

    # ---- the whole mixer stack (projections + pre-norm + residual) at the same B
    mixer = None
    if not args.no_mixer:
        mixer = run_mixer_stack(torch, dev, gen, cfg, gdn, abi, lib, pool, B, stream, barrier, dist, world, args,
                                hbm_peak)

    # ---- B sweep (1 GPU only): device tok/s and step-level HBM fraction
    sweep = {}
    for b in sweep_bs:
        if b == B:
            sweep[str(b)] = {"tok_s": value / world, "hbm_frac": roofline["step_frac"]}
            continue
        proj_s, out_s = buffers(b)
        gb = capture(b, proj_s, out_s)
        st = max(3, min(args.steps, int(2000 / max(b, 1))))
        msb = time_graph(gb, st, 3)
        step_bytes = N_LAYERS * (b * BYTES_PER_SEQ_LAYER + BYTES_PER_LAUNCH_CONST)
        sweep[str(b)] = {"tok_s": b * st / (msb / 1e3), "hbm_frac": step_bytes / (msb / st / 1e3) / 1e9 / hbm_peak}
        del gb, proj_s, out_s

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            os.sched_setaffinity(0, all_cpus)      # the CPU baseline uses every host core
            cpu = cpu_baseline(B)
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32 state, bf16 io", "data": "synthetic",
                "config": workload_config(B, world),
                "timed_step": "30 fused layer steps, gdn_layer_step_ex (layers 2-30 with GDN_STEP_TABLES_STABLE), "
                              "one CUDA graph; projections not included",
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": gpu_launches,
                "clocks": clk, "sweep": sweep or None, "mixer_stack": mixer, "prefill": prefill, "mixed": mixed,
                "sharded": sharded}
    if dist is not None:
        dist.barrier()
        del g
        dist.destroy_process_group()
    pool.close()
    if line is not None:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.hybrid_only:
        run_hybrid(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
