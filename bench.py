"""Benchmark of the Qwen3-30B-A3B sparse-MoE block on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload prefill|decode|skewed] [--ep peer|nccl]

A step is one forward of the MoE block (router, softmax/top-8, permute,
grouped gate/up GEMM + SwiGLU, grouped down GEMM + routing weight, combine)
over one batch of synthetic tokens:
  prefill (default): 8192 tokens per GPU (4 x 2048), seed 2;
  decode:            64 tokens, seed 1 (also reported as a sub-object of the
                     prefill line at N=1);
  skewed:            16384 tokens in all, split over the GPUs, Zipf(1.2)
                     router bias (strong scaling).
Weights are random N(0, 0.02) with the layer's real shapes (hidden 2048, 128
experts, top-8, intermediate 768); activations N(0, 1); bf16 storage, fp32
router and accumulation.  At N > 1 the block runs expert-parallel (E/N
experts per GPU, each GPU with its own 8192 tokens: weak scaling) with the
dispatch and combine exchanged over NVLink peer memory by library kernels
(--ep peer, default) or by NCCL all-to-all (--ep nccl).

`value`: CUDA-graph replay with the inputs resident.  `e2e`: the same batches
from page-locked host memory, copied in and back inside the timed region (at
N=1 through the host-batch block, copies overlapped with neighbouring
batches' blocks).  The line also carries the GEMM-1 roofline, the SM clocks
seen during the timed region, the CPU baseline (the oracle, N=1) and the
48-layer decoder stack's TTFT and decode tokens/s.

Prints ONE JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

# Token chunk of the host-buffer e2e calls (nkimoe_moe_block_host): one chunk
# per batch; the overlap is between successive batches.
E2E_CHUNK_TOKENS = 1 << 30

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of the
# dominant kernel (GEMM-1), from ncu captures of the 8192-token prefill and the
# 64-token decode workloads.
NCU_TRAFFIC_BYTES = {"prefill": 1.0739e9 + 92.66e6, "decode": 794.89e6 + 3.64e6}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="prefill", choices=["prefill", "decode", "skewed"],
                    help="prefill: 8192 tokens per GPU; decode: 64 tokens; skewed: 16384 tokens in all, split "
                         "over the GPUs, Zipf(1.2) router bias (strong scaling)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode sub-measurement")
    ap.add_argument("--no-skewed", action="store_true", help="skip the skewed-routing sub-measurement")
    ap.add_argument("--profile-once", action="store_true", help="one warm step only (for ncu launch lists)")
    ap.add_argument("--no-stack", action="store_true", help="skip the 48-layer decoder-stack TTFT / decode run")
    ap.add_argument("--stack-profile-layers", type=int, default=0,
                    help="with --profile-once: build a decoder stack of this many layers, prefill batch 8 x 512 "
                         "and run one eager decode step inside the NVTX range 'decode_step' (for ncu launch lists)")
    ap.add_argument("--ep-overlap", type=int, default=-1, choices=[-1, 0, 1, 2],
                    help="N > 1, peer exchange: -1 the library's choice (copy engines for prefill batches); 0 one block "
                         "after all rows arrived; 1 overlapped, SM stores on a side stream; 2 overlapped, copy engines")
    ap.add_argument("--ep-groups", type=int, default=0, help="N > 1, overlapped schedule: remote region groups (0 auto)")
    ap.add_argument("--ep-side-ctas", type=int, default=0,
                    help="N > 1, overlapped schedule: CTAs of the send / return kernels beside the GEMMs (0: library "
                         "default)")
    ap.add_argument("--gemm-schedule", type=int, default=None,
                    help="expert GEMM tile schedule (library option gemm_schedule; default: the library's)")
    ap.add_argument("--ep-replicas", type=int, default=-1,
                    help="N > 1, peer exchange: extra expert slots per rank for copies of hot experts, planned from "
                         "the routing of a calibration batch (-1: 2 for the skewed workload, 0 otherwise)")
    ap.add_argument("--ep", default="peer", choices=["peer", "nccl"],
                    help="N > 1: exchange over peer memory (library kernels) or NCCL all-to-all")
    return ap.parse_args()


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event (throttle) reasons during the timed region,
    polled through NVML every ~2 ms in a background thread (read-only
    queries), so that a timed region of tens of milliseconds still holds
    samples; falls back to ``nvidia-smi -lms 100`` when NVML is missing."""

    # NVML clock-event reason bits (nvmlClocksEventReason*)
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []  # (time, sm_mhz, max_mhz, set of reasons)
        self.t_start = self.t_end = None
        self._stop = threading.Event()
        self._nvml = None
        self.proc = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self._nvml = (pynvml, h)
            threading.Thread(target=self._poll_nvml, daemon=True).start()
            return
        except Exception:  # noqa: BLE001 - no NVML: use nvidia-smi
            self._nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", str(self.gpu),
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        threading.Thread(target=self._read_smi, daemon=True).start()

    def _poll_nvml(self):
        nv, h = self._nvml
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            except Exception:  # noqa: BLE001
                break
            self.rows.append((time.time(), float(sm), float(mx),
                              {n for b, n in self.REASONS.items() if bits & b}))
            time.sleep(0.002)

    def _read_smi(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.strip().split(",")]
            if len(parts) < 9:
                continue
            try:
                names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
                rs = {n for n, v in zip(names, parts[5:9]) if v.lower() in ("active", "1", "yes")}
                self.rows.append((time.time(), float(parts[1]), float(parts[2]), rs))
            except ValueError:
                continue

    def mark(self, start: bool):
        if start:
            self.t_start = time.time()
        else:
            self.t_end = time.time()

    def stop(self):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = list(self.rows)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"], "samples": 0}
        inwin = [r for r in rows if self.t_start and self.t_end and self.t_start <= r[0] <= self.t_end]
        use = inwin or rows
        mhz = sorted(r[1] for r in use)
        reasons = set()
        for r in use:
            reasons |= r[3]
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": max(r[2] for r in use), "reasons": sorted(reasons),
                "samples": len(use), "samples_in_timed_region": len(inwin),
                "source": "nvml" if self._nvml else "nvidia-smi"}


# ---------------------------------------------------------------- helpers
def algorithmic(wl, idx_np=None, tokens=None):
    """FLOPs and bytes of one block (``tokens`` of the workload, default all of
    them) and of its GEMM-1 launch."""
    import numpy as np
    T = wl.tokens if tokens is None else tokens
    H, I, E, K = wl.hidden, wl.intermediate, wl.experts, wl.top_k
    R = T * K
    u = len(np.unique(idx_np)) if idx_np is not None else E
    return {
        "block_flops": wl.flops * T / wl.tokens,
        "gemm1_flops": 2.0 * R * H * 2 * I,
        "gemm2_flops": 2.0 * R * I * H,
        # bytes that must move at least once: touched expert weights + activations in/out
        "gemm1_bytes": u * 2 * I * H * 2 + R * H * 2 + R * I * 2,
        "gemm2_bytes": u * H * I * 2 + R * I * 2 + R * H * 2,
        "block_bytes": u * wl.expert_bytes + E * H * 4 + 2 * T * H * 2 + T * K * 8,
        "unique_experts": int(u),
    }


def stage_events(torch):
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(13)]
    for e in evs:  # torch creates the CUDA event lazily, on its first record
        e.record()
    torch.cuda.synchronize()
    return evs


def set_stage_events(evs):
    import ctypes

    from nki_moe_b200 import _lib
    if evs is None:
        _lib.call("nkimoe_set_stage_events", None, 0)
        return
    arr = (ctypes.c_void_p * len(evs))(*[ctypes.c_void_p(e.cuda_event) for e in evs])
    _lib.call("nkimoe_set_stage_events", arr, len(evs))


# Stage events the library records (nkimoe_set_stage_events), in time order,
# and the names of the intervals between consecutive ones.
STAGE_ORDER = [0, 1, 2, 3, 4, 5, 6, 7]
STAGES = ["router", "topk", "permute", "gather", "gemm1_swiglu", "gemm2_scale", "combine"]
EP_STAGE_ORDER = [0, 1, 8, 9, 2, 3, 4, 5, 6, 10, 11, 12]  # one-block schedule (option ep_overlap 0)
EP_STAGES = ["router", "topk_and_rank_sort", "ep_send", "ep_wait", "permute", "gather", "gemm1_swiglu",
             "gemm2_scale", "combine_return", "ep_return_wait", "ep_sum"]
EPO_STAGE_ORDER = [0, 1, 2, 8, 9, 10, 11, 12]  # overlapped schedule (the default)
EPO_STAGES = ["router", "topk", "rank_sort", "own_tokens_first_half", "remote_groups",
              "own_tokens_second_half_and_return_wait", "ep_sum"]


def cpu_oracle_tokens_per_s(inp_cpu, wl, sample_tokens, repeat=1):
    """The oracle (numpy restatement of the reference CPU path) on a bounded
    token sample: router + top-8 + grouped expert FFNs + combine."""
    import numpy as np

    import oracle
    x = inp_cpu["x"][:sample_tokens]
    t0 = time.perf_counter()
    for _ in range(repeat):
        lg = oracle.router_logits(x, inp_cpu["router"]) + inp_cpu["router_bias"]
        idx, w = oracle.topk_softmax(lg, wl.top_k)
        oracle.experts_forward(x, inp_cpu["gate_up"], inp_cpu["down"], idx, w)
    dt = (time.perf_counter() - t0) / repeat
    return sample_tokens / dt, dt


def cpu_inputs(inp, torch):
    return {k: v.to(torch.bfloat16).float().cpu().numpy() if k != "router" and k != "router_bias"
            else v.float().cpu().numpy() for k, v in inp.items()}


def bind_to_gpu_cpus(gpu_index: int):
    """Run this process on the CPUs next to its GPU (NVML's affinity mask for
    the device), so that its page-locked host buffers are allocated in that
    socket's memory and its host<->device copies do not cross sockets.
    Returns the previous affinity (restored for the CPU legs), or None."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
        ncpu = os.cpu_count() or 1
        masks = pynvml.nvmlDeviceGetCpuAffinity(h, (ncpu + 63) // 64)
        cpus = {64 * i + b for i, m in enumerate(masks) for b in range(64) if (int(m) >> b) & 1 and 64 * i + b < ncpu}
        before = os.sched_getaffinity(0)
        if cpus and cpus != before:
            os.sched_setaffinity(0, cpus)
            return before
    except Exception:  # noqa: BLE001 - no NVML or no affinity support: leave the process where it is
        pass
    return None


def pin_cpu_threads():
    """Use every host core for the CPU legs, whatever the launcher set
    (torchrun exports OMP_NUM_THREADS=1): torch's intra-op pool and the BLAS
    pools numpy loaded."""
    import numpy as np  # noqa: F401
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(n)
    except Exception:  # noqa: BLE001 - no threadpoolctl: numpy keeps its pool
        pass
    return n


def cpu_threads():
    import numpy as np  # noqa: F401
    try:
        from threadpoolctl import threadpool_info
        n = max((i.get("num_threads", 1) for i in threadpool_info()), default=os.cpu_count())
    except Exception:
        n = os.cpu_count()
    return int(n or 1)


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the reference CPU path runs once, on rank 0
    import numpy as np  # noqa: F401
    import torch

    from nki_moe_b200.workloads import WORKLOADS, make_moe_inputs
    wl = WORKLOADS[{"prefill": "c3", "decode": "c2", "skewed": "c4"}[args.workload]]
    pin_cpu_threads()
    sample = wl.tokens if args.workload == "decode" else 1024
    inp = make_moe_inputs(wl, tokens=sample)
    cin = cpu_inputs(inp, torch)
    for _ in range(max(args.warmup, 0)):
        cpu_oracle_tokens_per_s(cin, wl, sample)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_oracle_tokens_per_s(cin, wl, sample)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    tps = sample / dt
    cores = cpu_threads()
    line = {
        "impl": "reference", "metric": "moe_block_tokens_per_s", "value": tps, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "strong" if args.workload == "skewed" else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.name,
                   "tokens_per_gpu": wl.tokens // args.gpus if args.workload == "skewed" else wl.tokens,
                   "hidden": wl.hidden, "experts": wl.experts,
                   "top_k": wl.top_k, "intermediate": wl.intermediate, "sample_tokens_per_step": sample},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{sample} tokens of the {wl.name} workload per step (numpy oracle, fp32)"},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cpu": {"os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads(),
                "model": _cpu_model()},
    }
    print(json.dumps(line), flush=True)


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# ---------------------------------------------------------------- B200 arm
def time_steps(torch, fn, steps, warmup, stream, world, evs=None, finish=None):
    """Device time per step over `steps` steps (CUDA events on `stream`, max
    over ranks).  `finish` (optional) runs after the last step, before the end
    event: it makes `stream` wait for work the steps left on other streams."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stage_ms = [0.0] * (len(STAGES))
    start.record(stream)
    for _ in range(steps):
        fn()
    if finish is not None:
        finish()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms, stage_ms


def measure_stages(torch, fn, steps, evs, graph_of=None, order=None):
    """Per-kernel durations from CUDA events that the library records between
    its launches on the launching stream, averaged over `steps` steps: the
    intervals between consecutive events of `order`.  With `graph_of`, the
    step is captured into a CUDA graph together with its event records and
    replayed, so the durations exclude CPU launch gaps."""
    order = order or STAGE_ORDER
    set_stage_events(evs)
    try:
        run = fn
        if graph_of is not None:
            run = graph_of(fn).replay
        acc = [0.0] * (len(order) - 1)
        for _ in range(steps):
            run()
            torch.cuda.synchronize()
            for i in range(len(order) - 1):
                acc[i] += evs[order[i]].elapsed_time(evs[order[i + 1]])
    finally:
        set_stage_events(None)
    return [a / steps for a in acc]


def measure_stack(torch, world=1, rank=0):
    """The full-stack configuration: random-init Qwen3-30B-A3B (48 layers),
    batch 8 x 512-token prompts, 128 greedy tokens.  TTFT is the prefill
    through the first token; decode steps replay one CUDA graph each.  With
    world > 1 the stack is expert-parallel: every rank holds the attention
    and E / world experts per layer and serves 8 / world of the sequences; the
    times are the maximum over ranks."""
    from nki_moe_b200.qwen_stack import Qwen3MoEConfig, Qwen3MoEStack

    cfg = Qwen3MoEConfig()
    B, S, new = 8, 512, 128
    Bl = B // world
    st = Qwen3MoEStack.random_init(cfg, seed=0, max_batch=Bl, max_seq=S + new, expert_parallel=world > 1)
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(0))[rank * Bl:(rank + 1) * Bl]
    st.generate(ids, 8)  # warm-up, graph capture
    _, t = st.generate(ids, new)
    ttft, dec = t["ttft_ms"], t["decode_ms"]
    if world > 1:
        v = torch.tensor([ttft, dec], device="cuda")
        torch.distributed.all_reduce(v, op=torch.distributed.ReduceOp.MAX)
        ttft, dec = float(v[0]), float(v[1])
    st.close()
    del st
    torch.cuda.empty_cache()
    steps = t["decode_steps"]
    return {"config": f"Qwen3-30B-A3B decoder stack, {cfg.num_hidden_layers} layers, random-init bf16 weights "
                      f"(router fp32); batch {B} x {S}-token prompts (uniform random ids, seed 0); {new} greedy "
                      f"tokens" + (f"; expert parallel over {world} GPUs, {Bl} sequences per GPU" if world > 1
                                   else ""),
            "ttft_ms": ttft, "decode_ms_per_step": dec / steps, "decode_tok_s": B * steps / (dec * 1e-3),
            "output_tok_s": B * new / ((ttft + dec) * 1e-3),
            "timing": "CUDA events; one CUDA graph replay per decode step" + (", max over ranks" if world > 1 else ""),
            "data": "synthetic"}


def ep_exchange_counts(torch, idx, world, rank, experts, block=None):
    """(token, rank) rows and (token, slot) pairs between the ranks of an
    expert-parallel step, from every rank's routing: rows[s][d] = tokens of
    rank s with an expert on rank d (each sent once), pairs[s][d] = their
    (token, slot) pairs.  With a peer block holding hot-expert replicas, slot
    (t, k) goes to the rank of holder t mod n_e of its expert, as the
    exchange sends it."""
    import torch.distributed as dist
    if block is not None and getattr(block, "replicas", None) is not None:
        il = idx.long()
        t = torch.arange(idx.shape[0], device=idx.device).unsqueeze(1)
        v = block.expert_slots.long()[il, t % block.slot_counts.long()[il]]
        dr = v // block.local_slots
    else:
        dr = idx.long() // (experts // world)
    hit = torch.zeros(idx.shape[0], world, dtype=torch.bool, device=idx.device)
    hit.scatter_(1, dr, True)
    mine = torch.stack([hit.sum(0), torch.bincount(dr.flatten(), minlength=world)]).to(torch.int64)
    allv = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allv, mine)
    m = torch.stack(allv).cpu()  # [src, 2, dst]
    return m[:, 0, :], m[:, 1, :]


def block_parity(torch, y, ref, idx=None, ref_idx=None, world=1):
    """Normwise error and cosine of an output against the single-GPU block's
    on the same tokens, and the tokens whose routing differs; max / min / sum
    over the ranks."""
    a, b = y.float(), ref.float()
    err = ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).reshape(1)
    cos = (torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0)).reshape(1)
    mis = torch.zeros(1, device=y.device)
    if idx is not None and ref_idx is not None:
        mis[0] = (idx != ref_idx).any(dim=1).sum().float()
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
        cos = -cos
        dist.all_reduce(cos, op=dist.ReduceOp.MAX)
        cos = -cos
        dist.all_reduce(mis, op=dist.ReduceOp.SUM)
    return {"normwise_max": float(err), "cosine_min": float(cos),
            "routing_mismatch_tokens": int(mis) if idx is not None else None,
            "pass": bool(float(err) <= 2e-2 and float(cos) >= 0.999 and (idx is None or int(mis) == 0))}


def run_b200(args):
    import numpy as np
    import torch

    from nki_moe_b200 import _lib, ops
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple
    from nki_moe_b200.workloads import WORKLOADS, make_moe_inputs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    _lib.load()
    _lib.set_option("ep_overlap", args.ep_overlap)
    _lib.set_option("ep_groups", args.ep_groups)
    if args.gemm_schedule is not None:
        _lib.set_option("gemm_schedule", args.gemm_schedule)
    if args.ep_side_ctas:
        _lib.set_option("ep_side_ctas", args.ep_side_ctas)
    if args.profile_once and args.stack_profile_layers > 0:
        from nki_moe_b200.qwen_stack import Qwen3MoEConfig, Qwen3MoEStack

        st = Qwen3MoEStack.random_init(Qwen3MoEConfig(num_hidden_layers=args.stack_profile_layers), seed=0,
                                       max_batch=8, max_seq=640)
        ids = torch.randint(0, st.cfg.vocab_size, (8, 512), generator=torch.Generator().manual_seed(0))
        st.prefill(ids)
        tok = torch.zeros(8, dtype=torch.int64, device="cuda")
        for _ in range(3):
            st.decode(tok, graph=False)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_step")
        st.decode(tok, graph=False)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        return
    hbm_gbs, tf_burst, tf_sus, peak_src = peaks()
    all_cpus = bind_to_gpu_cpus(local) if world > 1 else None
    sampler = ClockSampler(local)
    sampler.start()
    ep_peer = world > 1 and args.ep == "peer"

    def setup(wl):
        inp = make_moe_inputs(wl, device="cuda")
        moe = NKIMoESimple(wl.hidden, wl.intermediate, wl.experts, wl.top_k, device="cuda", dtype=torch.bfloat16)
        with torch.no_grad():
            moe.router.weight.copy_(inp["router"])
            moe.gate_up_proj.copy_(inp["gate_up"].to(torch.bfloat16))
            moe.down_proj.copy_(inp["down"].to(torch.bfloat16))
        if wl.zipf_s is not None:
            moe.router_bias = inp["router_bias"]
        x = inp["x"].to(torch.bfloat16)
        if wl.zipf_s is not None and world > 1:  # the batch is split over the ranks
            x = x.view(world, wl.tokens // world, wl.hidden)[rank].contiguous()
        elif world > 1:  # every rank has its own tokens (data-parallel shard)
            g = torch.Generator(device="cuda").manual_seed(wl.seed * 1000 + rank)
            x = torch.randn(wl.tokens, wl.hidden, generator=g, device="cuda").to(torch.bfloat16)
        return inp, moe, x

    def graph_of(fn):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
            fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    def max_over_ranks(vals):
        if world == 1:
            return list(vals)
        t = torch.tensor(list(vals), device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return t.tolist()

    def gather_ranks(v):
        if world == 1:
            return [v]
        t = torch.tensor([float(v)], device="cuda", dtype=torch.float64)
        out = [torch.empty_like(t) for _ in range(world)]
        torch.distributed.all_gather(out, t)
        return [float(o) for o in out]

    result = {}
    workloads = [args.workload]
    if args.workload == "prefill" and world == 1 and not args.no_decode:
        workloads.append("decode")
    if args.workload == "prefill" and not args.no_skewed:
        workloads.append("skewed")
    wl_key = {"prefill": "c3", "decode": "c2", "skewed": "c4"}
    for which in workloads:
        wl = WORKLOADS[wl_key[which]]
        inp, moe, x = setup(wl)
        T_local = x.shape[0]
        pe = moe.packed()
        rw, rb = moe.router.weight, moe.router_bias
        stream = torch.cuda.current_stream()
        # the single-GPU block on this rank's batch: routing (the algorithmic
        # byte count) and, at N > 1, the parity reference of the EP output
        y_one, idx_one, _ = ops.moe_block(x, rw, pe, wl.top_k, bias=rb, return_routing=True)
        alg = algorithmic(wl, idx_one.cpu().numpy(), tokens=T_local)
        block = None
        if world > 1:
            if ep_peer:
                from nki_moe_b200.ep_peer import PeerExpertParallelMoE, expert_load
                extra = args.ep_replicas if args.ep_replicas >= 0 else (2 if which == "skewed" else 0)
                load = None
                if extra > 0:
                    # the plan comes from another batch of the same distribution
                    # (its routing summed over the ranks), not the timed one
                    g_cal = torch.Generator(device="cuda").manual_seed(wl.seed * 7919 + 17 + rank)
                    x_cal = torch.randn(T_local, wl.hidden, generator=g_cal, device="cuda").to(torch.bfloat16)
                    _, idx_cal, _ = ops.moe_block(x_cal, rw, pe, wl.top_k, bias=rb, return_routing=True)
                    load = expert_load(idx_cal, wl.experts)
                    del x_cal, idx_cal
                # epochs counted on the device: the step replays as a CUDA graph
                block = PeerExpertParallelMoE.from_dense(moe, max_tokens=T_local, device_epochs=True,
                                                         extra_slots=extra, expected_load=load)
            else:
                from nki_moe_b200.ep import ExpertParallelMoE
                block = ExpertParallelMoE.from_dense(moe, torch.distributed.group.WORLD)
            fwd = lambda: block(x)  # noqa: E731
        else:
            fwd = lambda: ops.moe_block(x, rw, pe, wl.top_k, bias=rb)  # noqa: E731
        if args.profile_once:
            fwd()
            torch.cuda.synchronize()
            return
        # the NCCL exchange synchronises with the host (split sizes): eager
        use_graph = world == 1 or ep_peer
        run = graph_of(fwd).replay if use_graph else fwd
        if which == workloads[0]:  # clocks over the headline measurement's timed region
            sampler.mark(True)
        ms, _ = time_steps(torch, run, args.steps, max(args.warmup, 3), stream, world)
        if which == workloads[0]:
            sampler.mark(False)
        order, names = (EP_STAGE_ORDER, EP_STAGES) if ep_peer else (STAGE_ORDER, STAGES)
        st = st_o = ep_schedule = None
        n_stage_steps = max(5, min(args.steps, 20))
        if ep_peer:
            # the timed (overlapped) schedule's stages; then the one-block
            # schedule, whose stages isolate each kernel (GEMM-1 roofline,
            # exchange rates) -- every rank takes the same steps
            schedule = _lib.size_call("nkimoe_ep_peer_schedule", world, T_local)
            ep_schedule = {0: "one block", 1: "overlapped, SM stores", 2: "overlapped, copy engines"}[schedule]
            if schedule != 0:
                st_o = measure_stages(torch, fwd, n_stage_steps, stage_events(torch), graph_of, EPO_STAGE_ORDER)
            _lib.set_option("ep_overlap", 0)
            try:
                st = measure_stages(torch, fwd, n_stage_steps, stage_events(torch), graph_of, order)
            finally:
                _lib.set_option("ep_overlap", args.ep_overlap)
        elif world == 1:
            st = measure_stages(torch, fwd, n_stage_steps, stage_events(torch), graph_of if use_graph else None, order)
        tokens_total = T_local * world
        r = {"ms_per_step": ms, "tokens_per_s": tokens_total / (ms * 1e-3),
             "block_tflops": alg["block_flops"] * world / (ms * 1e-3) / 1e12,
             "block_gbs": alg["block_bytes"] * world / (ms * 1e-3) / 1e9, "alg": alg, "stages_ms": None}
        if ep_schedule is not None:
            r["ep_schedule"] = ep_schedule
        i1, i2 = names.index("gemm1_swiglu"), names.index("gemm2_scale")
        if st is not None:
            st_max = max_over_ranks(st)
            r["stages_ms"] = dict(zip(names, [round(v, 4) for v in st_max]))
            if world > 1:
                r["stages_ms_note"] = "per stage, the maximum over ranks of the rank's mean over steps"
        if st_o is not None:
            r["stages_ms_one_block"] = r["stages_ms"]
            r["stages_ms"] = dict(zip(EPO_STAGES, [round(v, 4) for v in max_over_ranks(st_o)]))
            r["stages_ms_note"] = ("per stage, the maximum over ranks of the rank's mean over steps; stages_ms: the "
                                   "timed overlapped schedule (sends and returns on a side stream beside the expert "
                                   "GEMMs); stages_ms_one_block: the one-block schedule, whose stages isolate the "
                                   "kernels (the roofline and exchange figures come from it)")
        if world > 1:
            rows, pairs = ep_exchange_counts(torch, idx_one, world, rank, wl.experts,
                                             block if ep_peer else None)
            if ep_peer and block.replicas is not None:
                _, pairs0 = ep_exchange_counts(torch, idx_one, world, rank, wl.experts)
                r["replicas"] = {
                    "extra_slots_per_rank": block.local_slots - wl.experts // world,
                    "copies": sum(len(h) - 1 for h in block.replicas[1]),
                    "max_holders": block.max_holders,
                    "rank_rows_max_over_mean_without": float(pairs0.sum(0).max() / pairs0.sum(0).float().mean()),
                    "plan": "greedy copies of the busiest rank's heaviest expert onto the least loaded rank, from "
                            "the routing of a separate calibration batch of the same distribution"}
            pairs_in = int(pairs[:, rank].sum())
            rows_out_remote = int(rows[rank].sum() - rows[rank, rank])
            rows_in_remote = int(rows[:, rank].sum() - rows[rank, rank])
            r["alg"]["gemm1_flops"] = 2.0 * pairs_in * wl.hidden * 2 * wl.intermediate
            r["alg"]["gemm2_flops"] = 2.0 * pairs_in * wl.intermediate * wl.hidden
            r["rank_rows_max_over_mean"] = float(pairs.sum(0).max() / pairs.sum(0).float().mean())
            if st is not None:
                d_bytes = rows_out_remote * (2 * wl.hidden + 8 * wl.top_k)
                r_bytes = rows_in_remote * 2 * wl.hidden
                t_send, t_ret = st[names.index("ep_send")], st[names.index("combine_return")]
                send_gbs = gather_ranks(d_bytes / (t_send * 1e-3) / 1e9)
                ret_gbs = gather_ranks(r_bytes / (t_ret * 1e-3) / 1e9)
                exposed = max_over_ranks([st[names.index("ep_send")] + st[names.index("ep_wait")] +
                                          st[names.index("ep_return_wait")] + st[names.index("ep_sum")]])[0]
                r["exchange"] = {
                    "dispatch_bytes_out_rank0": d_bytes, "return_bytes_out_rank0": r_bytes,
                    "send_gbs_min_over_ranks": min(send_gbs), "send_gbs_rank0": send_gbs[0],
                    "return_gbs_min_over_ranks": min(ret_gbs), "return_gbs_rank0": ret_gbs[0],
                    "nvlink_gbs_per_direction": 770.0,
                    "exposed_ms_max_over_ranks": exposed,
                        "note": "stores to peers over NVLink by the library's send and return-combine kernels, timed "
                            "in the one-block schedule (exposed_ms: its send, waits and final sum); the return stage "
                            "also holds the local rows' sums"}
        if st is not None and which in ("prefill", "skewed"):
            ach = gather_ranks(r["alg"]["gemm1_flops"] / (st[i1] * 1e-3) / 1e12)
            r["roofline"] = {"bound": "tensor", "kernel": "grouped_gemm_rows (gate/up + SwiGLU)",
                             "achieved": ach[0], "peak": tf_burst, "unit": "TFLOP/s", "frac": ach[0] / tf_burst,
                             "traffic": NCU_TRAFFIC_BYTES["prefill"] if world == 1 else None,
                             "peak_source": f"{peak_src} bf16 burst"}
            if world > 1:
                r["roofline"]["frac_min_over_ranks"] = min(ach) / tf_burst
                r["roofline"]["note"] = "rank 0's GEMM-1 over the (token, slot) pairs it received, per-GPU peak"
                step_flops = alg["block_flops"] * world
                r["roofline_step"] = {"achieved": step_flops / (ms * 1e-3) / 1e12, "peak": tf_burst * world,
                                      "frac": step_flops / (ms * 1e-3) / 1e12 / (tf_burst * world),
                                      "unit": "TFLOP/s", "note": "whole step, all ranks, against N x per-GPU peak"}
            a2 = gather_ranks(r["alg"]["gemm2_flops"] / (st[i2] * 1e-3) / 1e12)
            r["roofline_gemm2"] = {"bound": "tensor", "achieved": a2[0], "frac": a2[0] / tf_burst}
        elif st is not None:
            t = st[i1] * 1e-3
            r["roofline"] = {"bound": "hbm", "kernel": "grouped_gemm_weights (gate/up + SwiGLU)",
                             "achieved": alg["gemm1_bytes"] / t / 1e9, "peak": hbm_gbs, "unit": "GB/s",
                             "frac": alg["gemm1_bytes"] / t / 1e9 / hbm_gbs,
                             "traffic": NCU_TRAFFIC_BYTES["decode"], "peak_source": f"{peak_src} HBM copy"}
            blk = alg["block_bytes"] / (ms * 1e-3) / 1e9
            r["roofline_block"] = {"bound": "hbm", "achieved": blk, "frac": blk / hbm_gbs, "unit": "GB/s"}
        if which == "skewed" and world == 1:
            per_rank = np.bincount(idx_one.cpu().numpy().ravel() // (wl.experts // 8), minlength=8)
            r["rank_rows_max_over_mean_at_8"] = float(per_rank.max() / per_rank.mean())
        # parity of the expert-parallel output against the single-GPU block on
        # the same tokens (after the timed region; every rank takes part)
        if world > 1:
            if ep_peer:
                y_ep, idx_ep, _ = block(x, return_routing=True)
            else:
                y_ep, idx_ep = block(x), None
            r["parity"] = block_parity(torch, y_ep, y_one, idx_ep, idx_one if idx_ep is not None else None, world)
            r["parity"].update(vs="single-GPU nkimoe_moe_block on each rank's own batch", tokens=tokens_total,
                               bars="normwise <= 2e-2, cosine >= 0.999, no token routed differently")
            del y_ep
        # e2e through the public module API with pinned host buffers: successive
        # batches, each call's copy in overlapping the previous call's block and
        # its copy back the next call's block (two output buffers, one completion
        # event each)
        if not args.no_e2e:
            xh = x.reshape(1, *x.shape).cpu().pin_memory()
            outh = torch.empty_like(xh).pin_memory()
            outs = [outh[0], torch.empty_like(outh[0]).pin_memory()]
            dones = [torch.cuda.Event(), torch.cuda.Event()]
            n_e2e = [0]
            # the packed experts and the router's bf16 planes are made once, as
            # a serving loop keeps them
            e_split = ops.router_split(rw) if world == 1 else None

            def e2e_step():
                i = n_e2e[0] % 2
                n_e2e[0] += 1
                if world == 1:
                    ops.moe_block_host(xh[0], rw, pe, wl.top_k, bias=rb, out=outs[i],
                                       chunk_tokens=E2E_CHUNK_TOKENS, router_w_split=e_split, done=dones[i])
                elif ep_peer:
                    block.forward_host(xh[0], out=outs[i], done=dones[i])
                else:
                    xd = xh.to("cuda", non_blocking=True)
                    outs[i].copy_(block(xd[0]), non_blocking=True)
                    dones[i].record(stream)

            def e2e_finish():  # the timed region ends with the last copy back
                stream.wait_event(dones[(n_e2e[0] - 1) % 2])

            e_ms, _ = time_steps(torch, e2e_step, args.steps, max(args.warmup, 3), stream, world,
                                 finish=e2e_finish)
            r["e2e"] = {"value": tokens_total / (e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e_ms,
                        "h2d_bytes_per_step": xh.numel() * xh.element_size() * world,
                        "d2h_bytes_per_step": outh.numel() * outh.element_size() * world,
                        "path": ("ops.moe_block_host (nkimoe_moe_block_host)" if world == 1 else
                                 "PeerExpertParallelMoE.forward_host" if ep_peer else
                                 "copy in, ExpertParallelMoE, copy back") +
                                " on page-locked host batches: each batch copied in, through the block and copied "
                                "back, a batch's copies overlapping its neighbours' blocks"}
        if not args.no_cpu_baseline and rank == 0:
            # the oracle on this rank's whole batch, repeated to about 10 s of
            # CPU work (3 s for the sub-workloads), on every host core
            if all_cpus:
                os.sched_setaffinity(0, all_cpus)
            pin_cpu_threads()
            cin = cpu_inputs(inp, torch)
            cin["x"] = x.float().cpu().numpy()
            target = 10.0 if which == workloads[0] else 3.0
            _, one = cpu_oracle_tokens_per_s(cin, wl, T_local)
            rep = max(1, min(int(target / max(one, 1e-3)) + 1, int(30.0 / max(one, 1e-3))))
            tps, dt = cpu_oracle_tokens_per_s(cin, wl, T_local, repeat=rep)
            r["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
                                 "sample": f"the {T_local}-token {wl.name} batch"
                                           f"{' of rank 0' if world > 1 else ''} x {rep} (numpy oracle, fp32), "
                                           f"{dt * rep:.1f} s"}
            if all_cpus:
                bind_to_gpu_cpus(local)
        if world > 1:
            # the other ranks wait for rank 0's CPU leg on the rendezvous store
            # (a blocking socket read), not in a collective whose host threads
            # spin and would take cores from the CPU baseline
            store = torch.distributed.distributed_c10d._get_default_store()
            key = f"bench_cpu_leg_done_{which}"
            if rank == 0:
                store.set(key, "1")
            else:
                store.wait([key])
            torch.distributed.barrier()
        result[which] = r
        if block is not None and hasattr(block, "close"):
            block.close()
        del moe, inp, x, block, y_one, idx_one
        torch.cuda.empty_cache()

    sampler.stop()
    clocks = sampler.summary()
    main_key = workloads[0]
    m = result[main_key]
    wl = WORKLOADS[wl_key[main_key]]
    # this library's kernels per step: single GPU 9 (router GEMM, top-k, 3
    # permutation, gather, 2 GEMMs, combine); EP over peer memory 19 (+ epoch,
    # destinations, 3 rank-sort, send, 2 waits, mask, final sum); EP over NCCL
    # 17 of ours (NCCL's own kernels not counted)
    launches_per_step = 9 if world == 1 else (19 if ep_peer else 17)
    timing = ("CUDA graph replay, CUDA events" + (", max over ranks" if world > 1 else "")) if (world == 1 or ep_peer) \
        else "eager, CUDA events, max over ranks"
    line = {
        "metric": "moe_block_tokens_per_s", "value": m["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": m["ms_per_step"],
        "higher_is_better": True, "scaling": "strong" if main_key == "skewed" else "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": wl.name,
                   "tokens_per_gpu": wl.tokens // world if main_key == "skewed" else wl.tokens,
                   "hidden": wl.hidden, "experts": wl.experts,
                   "top_k": wl.top_k, "intermediate": wl.intermediate,
                   "parallelism": (f"ep{world}-{args.ep}" + ({-1: "-auto", 0: "-one-block", 1: "-overlapped-sm",
                                                             2: "-overlapped-copy-engines"}[args.ep_overlap]
                                                            if ep_peer else "")) if world > 1 else "single",
                   "l2": "inputs larger than L2 (1.21 GB of expert weights read per step)",
                   "timing": timing},
        "roofline": m.get("roofline"),
        "cpu_baseline": m.get("cpu_baseline"),
        "e2e": m.get("e2e"),
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "block_tflops": m["block_tflops"],
        "stages_ms": m["stages_ms"],
    }
    for k in ("roofline_gemm2", "roofline_step", "exchange", "parity", "stages_ms_note", "stages_ms_one_block",
              "ep_schedule"):
        if k in m:
            line[k] = m[k]
    if "rank_rows_max_over_mean" in m:
        line["rank_rows_max_over_mean"] = m["rank_rows_max_over_mean"]
    if "decode" in result and main_key != "decode":
        d = result["decode"]
        line["decode"] = {"workload": WORKLOADS["c2"].name, "tokens_per_s": d["tokens_per_s"],
                          "ms_per_step": d["ms_per_step"], "roofline": d.get("roofline"),
                          "roofline_block": d.get("roofline_block"), "stages_ms": d["stages_ms"],
                          "e2e": d.get("e2e"), "cpu_baseline": d.get("cpu_baseline"),
                          "unique_experts": d["alg"]["unique_experts"]}
    if "skewed" in result and main_key != "skewed":
        d = result["skewed"]
        line["skewed"] = {"workload": WORKLOADS["c4"].name, "tokens_total": WORKLOADS["c4"].tokens,
                          "tokens_per_gpu": WORKLOADS["c4"].tokens // world, "scaling": "strong",
                          "tokens_per_s": d["tokens_per_s"], "ms_per_step": d["ms_per_step"],
                          "block_tflops": d["block_tflops"],
                          "frac_of_n_x_peak": d["block_tflops"] / (tf_burst * world),
                          "rank_rows_max_over_mean": d.get("rank_rows_max_over_mean",
                                                           d.get("rank_rows_max_over_mean_at_8")),
                          "roofline": d.get("roofline"), "stages_ms": d["stages_ms"],
                          "stages_ms_one_block": d.get("stages_ms_one_block"), "ep_schedule": d.get("ep_schedule"),
                          "parity": d.get("parity"), "replicas": d.get("replicas"),
                          "exchange": d.get("exchange"), "e2e": d.get("e2e"), "cpu_baseline": d.get("cpu_baseline")}
    if not args.no_stack and (world == 1 or 8 % world == 0):
        line["stack"] = measure_stack(torch, world, rank)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
