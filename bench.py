#!/usr/bin/env python
"""Benchmark: slot_murmurate forward + backward tokens/s on B200.

Workload: B=1, H=16, N=8192, d=64, M=256, R=3, k=7,
non-causal, fp16, the inputs of BASELINE configs[1] (q ~ N(0,1), slots_k ~
N(0,1), slots_v = 0) plus grad_out ~ N(0,1) for the backward. One step = one
forward and one backward pass over that batch. With N GPUs (torchrun, one
process per GPU) every rank runs its own batch of 16 (batch, head) pairs —
(b,h) pairs are independent, so there is no collective on the data path —
and ``value`` is all ranks' tokens divided by the slowest rank's time
(weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line. ``value`` is measured with the inputs resident
in HBM, the step replayed from a CUDA graph, L2 flushed (a read-modify-write kernel over 256 MiB)
before every timed step and CUDA events around each step. ``e2e`` is the same
metric through the public API for host-resident tensors
(murmurative_attention_b200.slot_murmurate_host_step, the C ABI's
murm_slot_murmurate_host_step) with pinned host buffers: every step copies q,
slots and grad_out to the device and copies out, indices, weights and the
three gradients back, pipelined over groups of (batch, head) pairs so the
copies overlap the kernels. ``e2e_autograd`` is the same through
slot_murmurate + autograd backward on device tensors copied in and out.
``roofline`` covers the kernel with the largest device time, timed with CUDA
events recorded on its own launch stream. Two more BASELINE configurations run
at the same N: ``strong`` is configs[2] (bf16 causal, 128 (batch, head) pairs)
as one global problem split over the ranks (strong scaling, outputs gathered
and checked against one GPU's run), ``layer`` is configs[3], the data-parallel
layer training step with its NCCL gradient all-reduce inside the timed region. The rows past the
hot path are measured in the same run: ``sp`` (sequence parallelism over the ranks, one NCCL
all-reduce of the slot sums per round), ``surface`` (the reference's 6-argument op with mask and
position bias) and ``decode`` (the streaming decode step).
``--impl reference`` times the reference's CPU path (the oracle port, which
runs the reference.py operations) on the host cores, whole steps of the
workload.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "slot_murmurate fwd+bwd tokens/s at N=8192, 1/2/4/8 B200; % of roofline"
WL = dict(B=1, H=16, N=8192, D=64, M=256, R=3, causal=False)
DTYPE = torch.float16  # --dtype bf16 switches the north-star workload to bfloat16 inputs
DTYPE_NAME = "fp16"
ESIZE = 2


def workload_config(extra=None):
    cfg = {"workload": f"northstar: BASELINE configs[1] inputs ({DTYPE_NAME} q~N(0,1) [1,16,8192,64], slots_k~N(0,1) "
                       "[1,16,256,64], slots_v=0) with backward (grad_out~N(0,1)); R=3, k=7, non-causal",
           "batch_per_rank": WL["B"], "heads": WL["H"], "tokens": WL["N"], "head_dim": WL["D"], "slots": WL["M"],
           "rounds": WL["R"], "top_k": 7, "causal": WL["causal"],
           "l2": "flushed before every timed step by a kernel reading and writing 256 MiB (inputs 16 MiB < 126 MB L2)"}
    if extra:
        cfg.update(extra)
    return cfg


def algorithmic_bytes():
    """Every tensor touched once (fwd: q in, out/idx/w out; bwd: q, grad_out in, grad_q out;
    slots read and written once per direction)."""
    BH, N, D, M = WL["B"] * WL["H"], WL["N"], WL["D"], WL["M"]
    per_token = 5 * D * ESIZE + 7 * 8 + 7 * 4
    return BH * N * per_token + BH * 6 * M * D * ESIZE


def select_flops_per_round():
    return 2 * WL["M"] * WL["D"] * WL["B"] * WL["H"] * WL["N"]


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return dict(hbm_gbs=j["hbm_gbs"], bf16_tflops=j["bf16_tflops"],
                    bf16_tflops_sustained=j.get("bf16_tflops_sustained"), source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, source="fallback")


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons while the timed steps run. NVML is read every 0.5 ms from a
    thread (reads only: the timed region is a few milliseconds, far shorter than nvidia-smi's
    sampling period); the interpreter's thread switch interval is cut to 0.1 ms meanwhile, so the
    sampler is not held off by the timing loop for the default 5 ms. Without NVML, nvidia-smi every
    100 ms. Any failure only drops the record."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index):
        self.proc = None
        self.thread = None
        self.dev = device_index
        self.samples = []  # (sm MHz, reason names)
        self.max_mhz = None
        self.halt = threading.Event()
        self.switch = None

    def _uuid(self):
        return "GPU-" + str(torch.cuda.get_device_properties(self.dev).uuid)

    def _start_nvml(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByUUID(self._uuid())
        except Exception:  # older bindings take bytes
            h = pynvml.nvmlDeviceGetHandleByUUID(self._uuid().encode())
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        bits = ((pynvml.nvmlClocksEventReasonHwSlowdown, "hw_slowdown"),
                (pynvml.nvmlClocksEventReasonHwThermalSlowdown, "hw_thermal_slowdown"),
                (pynvml.nvmlClocksEventReasonSwThermalSlowdown, "sw_thermal_slowdown"),
                (pynvml.nvmlClocksEventReasonSwPowerCap, "sw_power_cap"))

        def run():
            try:
                while not self.halt.is_set():
                    sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    mask = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((sm, tuple(n for b, n in bits if mask & b)))
                    time.sleep(0.0005)
            except Exception:
                pass
            finally:
                try:
                    pynvml.nvmlShutdown()
                except Exception:
                    pass

        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()

    def start(self):
        self.switch = sys.getswitchinterval()
        sys.setswitchinterval(1e-4)
        try:
            self._start_nvml()
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self._uuid(), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.switch is not None:
            sys.setswitchinterval(self.switch)
        try:
            return self._stop()
        except Exception:
            return None

    def _stop(self):
        if self.thread is not None:
            self.halt.set()
            self.thread.join(timeout=5)
            if not self.samples:
                return None
            sm = [x for x, _ in self.samples]
            reasons = sorted({n for _, ns in self.samples for n in ns})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz, "samples": len(sm),
                    "reasons": reasons, "source": "nvml, every 0.5 ms"}
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for nm, v in zip(self.NAMES, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons), "source": "nvidia-smi, every 100 ms"}


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------
class AbiStep:
    """One fwd+bwd step through the C ABI with preallocated device buffers."""

    def __init__(self, q, sk, sv, go, rounds=WL["R"], causal=WL["causal"]):
        from murmurative_attention_b200 import _lib, ops
        self._lib = _lib
        self.lib = _lib.load_library()
        B, H, N, D = q.shape
        self.shape = ops._make_shape(q, sk.shape[2], rounds, 7, causal, 0.9, 0.15, None)
        saved_b, fws_b, bws_b = ops.slot_murmurate_sizes(self.shape)
        dev = q.device
        self.keep = dict(q=q, sk=sk, sv=sv, go=go)
        self.out = torch.empty_like(q)
        self.idx = torch.empty(B, H, N, 7, dtype=torch.int64, device=dev)
        self.w = torch.empty(B, H, N, 7, dtype=torch.float32, device=dev)
        self.saved = torch.empty(saved_b, dtype=torch.uint8, device=dev)
        self.fws = torch.empty(fws_b, dtype=torch.uint8, device=dev)
        self.bws = torch.empty(bws_b, dtype=torch.uint8, device=dev)
        self.gq = torch.empty_like(q)
        self.gsk = torch.empty_like(sk)
        self.gsv = torch.empty_like(sv)
        S = ops._strides
        self.fargs = _lib.FwdArgs(self.shape, q.data_ptr(), S(q), sk.data_ptr(), S(sk), sv.data_ptr(), S(sv),
                                  self.out.data_ptr(), S(self.out), self.idx.data_ptr(), self.w.data_ptr(),
                                  self.saved.data_ptr(), saved_b, self.fws.data_ptr(), fws_b)
        self.bargs = _lib.BwdArgs(self.shape, q.data_ptr(), S(q), go.data_ptr(), S(go), None,
                                  self.saved.data_ptr(), saved_b, self.gq.data_ptr(), S(self.gq),
                                  self.gsk.data_ptr(), S(self.gsk), self.gsv.data_ptr(), S(self.gsv),
                                  self.bws.data_ptr(), bws_b)

    def __call__(self):
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        self._lib.check(self.lib.murm_slot_murmurate_fwd(ctypes.byref(self.fargs), st))
        self._lib.check(self.lib.murm_slot_murmurate_bwd(ctypes.byref(self.bargs), st))


def make_inputs(device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    B, H, N, D, M = WL["B"], WL["H"], WL["N"], WL["D"], WL["M"]
    q = torch.randn(B, H, N, D, generator=g, device=device).to(DTYPE)
    sk = torch.randn(B, H, M, D, generator=g, device=device).to(DTYPE)
    sv = torch.zeros(B, H, M, D, device=device, dtype=DTYPE)
    go = torch.randn(B, H, N, D, generator=g, device=device).to(DTYPE)
    return q, sk, sv, go


def graph_of(step):
    """The step replayed from a CUDA graph (no host launch overhead in the timed region), or the
    step itself when capture fails."""
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        g.replay()
        torch.cuda.synchronize()
        return g.replay, g
    except Exception as e:  # noqa: BLE001
        print(f"[bench] CUDA graph capture failed, timing eager launches: {e}", file=sys.stderr)
        return step, None


def flush_l2(buf):
    """Evict L2 before a timed step: a kernel that reads and writes every element of a 256 MiB
    buffer (twice the 126 MB L2). A cudaMemset of the buffer (tensor.zero_()) is not enough: its
    writes did not displace the step's inputs from L2 (measured: the first forward launch read
    5 of its 16.8 MB of q from DRAM after one)."""
    buf.add_(1.0)


def time_steps(fn, steps, flush_buf):
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush_l2(flush_buf)
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def run_ours(args):
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from murmurative_attention_b200 import _lib, slot_murmurate

    q, sk, sv, go = make_inputs(dev, seed=1000 + rank)
    step = AbiStep(q, sk, sv, go)
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=dev)
    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()

    # launches per step (counted by the library)
    n0 = _lib.kernel_launches()
    step()
    torch.cuda.synchronize()
    launches_per_step = _lib.kernel_launches() - n0

    # replay the step from a CUDA graph (no host launch overhead in the timed region)
    fn, graph = (step, None) if args.no_graph else graph_of(step)
    graph_used = graph is not None
    for _ in range(args.warmup):
        fn()
    barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    times = time_steps(fn, args.steps, flush)
    clk = clocks.stop()
    barrier(world)
    total_ms = max_over_ranks(sum(times), world)
    ms_per_step = total_ms / args.steps
    tokens_per_step = WL["B"] * WL["N"] * world
    value = tokens_per_step / (ms_per_step / 1e3)

    # per-kernel device time (eager launches, events on the launch stream)
    prof_steps = min(args.steps, 20)
    _lib.profile_begin()
    for _ in range(prof_steps):
        flush_l2(flush)
        step()
    torch.cuda.synchronize()
    prof = _lib.profile_end()

    # end to end through the public API with host buffers
    e2e = run_e2e_host(q, sk, sv, go, min(args.steps, 20), args.warmup, flush, world)
    e2e_autograd = run_e2e(q, sk, sv, go, min(args.steps, 20), args.warmup, flush, slot_murmurate, world)

    # the other BASELINE configurations at this N (every rank takes the same collective steps)
    strong = None if args.skip_strong else strong_leg(args, world, rank, dev, flush)
    layer = None if args.skip_layer else layer_leg(args, world, rank, dev, flush)
    sp = surface = decode = None
    if not args.skip_widening:  # the rows past the hot path, measured in the same run
        sp = sp_leg(args, world, rank, dev, flush)
        surface = surface_leg(args, dev, flush)
        decode = decode_leg(args, dev, flush)

    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    peaks = load_peaks()
    roof = roofline(prof, prof_steps, peaks)
    # whole-step roofline (every tensor touched once; the select GEMM on the tensor cores)
    t_hbm = algorithmic_bytes() / (peaks["hbm_gbs"] * 1e9)
    t_tc = WL["R"] * select_flops_per_round() / (peaks["bf16_tflops"] * 1e12)
    t_roof = max(t_hbm, t_tc)
    step_roof = {"t_roof_us": round(t_roof * 1e6, 2), "bound": "hbm" if t_hbm >= t_tc else "tensor",
                 "algorithmic_bytes": algorithmic_bytes(), "select_flops": WL["R"] * select_flops_per_round(),
                 "frac": round(t_roof / (ms_per_step / 1e3), 4),
                 "note": "T_roof = max(bytes/HBM, select FLOPs/tensor peak) per rank, measured peaks"}
    line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": DTYPE_NAME, "data": "synthetic",
            "config": workload_config({"parallelism": f"(batch,head)-sharded weak scaling, {world} rank(s)",
                                       "timing": "CUDA graph replay" if graph_used else "eager launches"}),
            "roofline": roof, "step_roofline": step_roof, "e2e": e2e, "e2e_autograd": e2e_autograd,
            "strong": strong, "layer": layer, "sp": sp, "surface": surface, "decode": decode,
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clk,
            "kernels": {k: {"launches_per_step": v[0] / prof_steps, "ms_per_step": round(v[1] / prof_steps, 5)}
                        for k, v in sorted(prof.items(), key=lambda kv: -kv[1][1])}}
    if world == 1 and not args.skip_cpu:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


CONFIG3 = dict(B=8, H=16, N=4096, D=64, M=256, R=3, causal=True)


def strong_leg(args, world, rank, dev, flush):
    """BASELINE configs[2] as ONE global problem split over the ranks by (batch, head) pair (strong
    scaling): bf16 causal, q ~ N(0,1) [8,16,4096,64], slots_k ~ N(0,1)/8, slots_v ~ N(0,0.02),
    grad_out ~ N(0,1), R=3, fwd+bwd. Every rank draws the same global inputs, runs its contiguous
    share of the 128 pairs (distributed.local_pairs; pairs are independent, so no collective is
    on the data path) and the step time is the slowest rank's. After timing, the indices and
    outputs are gathered (distributed.gather_pairs, NCCL all-gather) and rank 0 compares them with
    the whole problem run on its own GPU."""
    from murmurative_attention_b200.distributed import gather_pairs, local_pairs
    C = CONFIG3
    g = torch.Generator(device=dev).manual_seed(6000)
    tok = (C["B"], C["H"], C["N"], C["D"])
    slot = (C["B"], C["H"], C["M"], C["D"])
    q = torch.randn(*tok, generator=g, device=dev).to(torch.bfloat16)
    sk = (torch.randn(*slot, generator=g, device=dev) / 8).to(torch.bfloat16)
    sv = (torch.randn(*slot, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    go = torch.randn(*tok, generator=g, device=dev).to(torch.bfloat16)
    loc = [local_pairs(t, world, rank).contiguous() for t in (q, sk, sv, go)]
    step = AbiStep(*loc, rounds=C["R"], causal=C["causal"])
    for _ in range(args.warmup):
        step()
    fn, graph = graph_of(step)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    times = time_steps(fn, args.steps, flush)
    barrier(world)
    ms = max_over_ranks(sum(times), world) / args.steps
    step()  # the outputs of one plain step, for the check
    torch.cuda.synchronize()
    check = {"ranks": world}
    if world > 1:
        idx_all = gather_pairs(step.idx, C["B"], C["H"])
        out_all = gather_pairs(step.out, C["B"], C["H"])
        if rank == 0:
            whole = AbiStep(q, sk, sv, go, rounds=C["R"], causal=C["causal"])
            whole()
            torch.cuda.synchronize()
            same = (idx_all == whole.idx).all(-1)
            diff = (out_all.float() - whole.out.float()).abs()[same]
            check.update({"rows_with_equal_indices": round(float(same.float().mean()), 6),
                          "max_abs_out_diff_on_equal_rows": float(diff.max()) if diff.numel() else None,
                          "against": "the whole 128-pair problem run on rank 0's GPU alone"})
            del whole
    else:
        check["against"] = "one rank: the run is the whole problem"
    tokens = C["B"] * C["N"]
    return {"workload": "BASELINE configs[2]: bf16 causal [8,16,4096,64], sk~N(0,1)/8, sv~N(0,0.02), R=3, "
                        "fwd+bwd, 128 (batch,head) pairs split contiguously over the ranks",
            "value": round(tokens / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 5),
            "scaling": "strong", "pairs_per_rank": int(loc[0].shape[1]),
            "timing": "CUDA graph replay" if graph is not None else "eager launches", "check": check}


def layer_leg(args, world, rank, dev, flush):
    """the MurmurativeAttention layer training step, bf16, data parallel:
    every rank trains on its own 2 sequences of 8192 tokens (16 sequences at 8 GPUs) and the
    parameter gradients are averaged over NCCL while the backward runs (one all-reduce per
    parameter, started by autograd hooks: q_proj and o_proj weights 2 MiB each, slot embeddings
    0.5 MiB, bf16). One step = forward, mean-square loss, backward, gradient average, SGD update.
    The collective's cost is also timed alone (the same three all-reduces back to back)."""
    from murmurative_attention_b200 import MurmurativeAttention
    from murmurative_attention_b200.training import GradientAverager, dp_train_step
    L = LAYER
    torch.manual_seed(0)  # the same initial parameters on every rank
    layer = MurmurativeAttention(L["dim"], L["heads"], L["slots"], rounds=L["R"]).to(dev, torch.bfloat16)
    with torch.no_grad():
        layer.q_proj.weight.normal_(0.0, L["dim"] ** -0.5)
        layer.o_proj.weight.normal_(0.0, L["dim"] ** -0.5)
        layer.slot_embeddings.normal_(0.0, 1.0)
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    x = torch.randn(L["B"], L["N"], L["dim"], device=dev, dtype=torch.bfloat16, generator=g)
    opt = torch.optim.SGD(layer.parameters(), lr=1e-3)
    avg = GradientAverager(layer.parameters())
    for _ in range(args.warmup):
        dp_train_step(layer, x, opt, avg)
    torch.cuda.synchronize()
    barrier(world)
    times = time_steps(lambda: dp_train_step(layer, x, opt, avg), args.steps, flush)
    barrier(world)
    ms = max_over_ranks(sum(times), world) / args.steps
    avg.remove()
    grads = [p.grad for p in layer.parameters() if p.grad is not None]
    coll = {"collective": "none (one rank)"}
    if world > 1:
        import torch.distributed as dist

        def reduce_all():
            for t in grads:
                dist.all_reduce(t)
        for _ in range(3):
            reduce_all()
        torch.cuda.synchronize()
        barrier(world)
        ar = time_steps(reduce_all, args.steps, flush)
        ar_ms = max_over_ranks(sum(ar), world) / args.steps
        nbytes = sum(t.numel() * t.element_size() for t in grads)
        coll = {"collective": f"NCCL all_reduce (sum) of the {len(grads)} parameter gradients, "
                              f"{nbytes / 2**20:.2f} MiB bf16 per step, overlapped with the backward",
                "allreduce_ms_alone": round(ar_ms, 5), "share_of_step_if_not_overlapped": round(ar_ms / ms, 4)}
    tokens = world * L["B"] * L["N"]
    return {"workload": "layer (BASELINE configs[3]): dim 1024, heads 16 (d=64), M=256, R=3, k=7, "
                        "x~N(0,1) [2 per rank,8192,1024], q_proj/o_proj ~N(0,1/1024), slot_embeddings ~N(0,1); SGD",
            "value": round(tokens / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 5),
            "scaling": "weak", "global_batch": world * L["B"], "seq_len": L["N"], "parallelism": f"dp{world}",
            **coll}


def roofline(prof, prof_steps, peaks):
    if not prof:
        return None
    name, (launches, total) = max(prof.items(), key=lambda kv: kv[1][1])
    avg_ms = total / launches
    # DRAM bytes per launch cannot be read without a profiler: they come from the committed
    # ncu capture of the same kernel (static, labelled as such), not from this run
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic_northstar.json")
    if os.path.exists(tpath) and DTYPE_NAME == "fp16":
        with open(tpath) as f:
            traffic = json.load(f).get(name)
    traffic_source = ("static: dram__bytes_read.sum + dram__bytes_write.sum per launch from the ncu capture "
                      "recorded in profiles/traffic_northstar.json, not measured in this run"
                      if DTYPE_NAME == "fp16" else "no ncu capture of the bf16 kernels recorded")
    if name.startswith("select"):
        # the forward runs all R rounds in one launch (one launch per round on the fallback path)
        rounds_per_launch = WL["R"] * prof_steps / launches
        flops = select_flops_per_round() * rounds_per_launch
        achieved = flops / (avg_ms / 1e3) / 1e12
        return {"kernel": name, "bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4), "traffic": traffic,
                "peak_source": f"{peaks['source']} (burst dense bf16)",
                "work_per_launch": f"select GEMM 2*M*d*tokens per round x {rounds_per_launch:g} rounds = {flops:.4g} FLOP",
                "avg_launch_ms": round(avg_ms, 5), "launches": launches, "traffic_source": traffic_source}
    # memory-bound kernels: algorithmic bytes of the whole step spread over its launches
    per_launch = algorithmic_bytes() / (launches / prof_steps)
    achieved = per_launch / (avg_ms / 1e3) / 1e9
    return {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic, "traffic_source": traffic_source,
            "peak_source": f"{peaks['source']} copy bandwidth", "avg_launch_ms": round(avg_ms, 5),
            "launches": launches}


def run_e2e_host(q, sk, sv, go, steps, warmup, flush, world, groups=0):
    from murmurative_attention_b200 import slot_murmurate_host_step
    host = {k: t.detach().cpu().contiguous().pin_memory() for k, t in dict(q=q, sk=sk, sv=sv, go=go).items()}
    B, H, N, D = host["q"].shape
    outs = (torch.empty_like(host["q"]).pin_memory(), torch.empty(B, H, N, 7, dtype=torch.int64).pin_memory(),
            torch.empty(B, H, N, 7).pin_memory(), torch.empty_like(host["q"]).pin_memory(),
            torch.empty_like(host["sk"]).pin_memory(), torch.empty_like(host["sv"]).pin_memory())

    def one():
        slot_murmurate_host_step(host["q"], host["sk"], host["sv"], host["go"], rounds=WL["R"], causal=WL["causal"],
                                 groups=groups, outputs=outs)

    for _ in range(max(warmup, 1)):
        one()
    torch.cuda.synchronize()
    barrier(world)
    times = time_steps(one, steps, flush)
    total = max_over_ranks(sum(times), world)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in outs)
    ms = total / steps
    return {"value": round(WL["B"] * WL["N"] * world / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "path": "murmurative_attention_b200.slot_murmurate_host_step (C ABI murm_slot_murmurate_host_step): "
                    "pinned host buffers, copies pipelined with the kernels over groups of (b,h) pairs"}


def run_e2e(q, sk, sv, go, steps, warmup, flush, op, world):
    host = {k: t.detach().cpu().pin_memory() for k, t in dict(q=q, sk=sk, sv=sv, go=go).items()}
    dev = q.device
    outs = None

    def one():
        nonlocal outs
        qd = host["q"].to(dev, non_blocking=True).requires_grad_(True)
        skd = host["sk"].to(dev, non_blocking=True).requires_grad_(True)
        svd = host["sv"].to(dev, non_blocking=True).requires_grad_(True)
        god = host["go"].to(dev, non_blocking=True)
        out, idx, w = op(qd, skd, svd, rounds=WL["R"], causal=WL["causal"])
        out.backward(god)
        res = (out.detach(), idx, w.detach(), qd.grad, skd.grad, svd.grad)
        if outs is None:
            outs = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in res]
        for h, t in zip(outs, res):
            h.copy_(t, non_blocking=True)

    for _ in range(max(warmup, 1)):
        one()
    torch.cuda.synchronize()
    barrier(world)
    times = time_steps(one, steps, flush)
    total = max_over_ranks(sum(times), world)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in outs)
    ms = total / steps
    return {"value": round(WL["B"] * WL["N"] * world / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "path": "murmurative_attention_b200.slot_murmurate + autograd backward, pinned host buffers"}


# ---------------------------------------------------------------------------
# CPU: the reference path (oracle port of reference.py) on the host cores
# ---------------------------------------------------------------------------
def cpu_sample_step(heads, seed=0):
    import oracle
    g = torch.Generator().manual_seed(seed)
    N, D, M = WL["N"], WL["D"], WL["M"]
    q = torch.randn(1, heads, N, D, generator=g).to(DTYPE).float().requires_grad_(True)
    sk = torch.randn(1, heads, M, D, generator=g).to(DTYPE).float().requires_grad_(True)
    sv = torch.zeros(1, heads, M, D, requires_grad=True)
    go = torch.randn(1, heads, N, D, generator=g).to(DTYPE).float()

    def step():
        q.grad = sk.grad = sv.grad = None
        out, idx, w = oracle.slot_murmurate(q, sk, sv, rounds=WL["R"], causal=WL["causal"], tie_rule="topk")
        out.backward(go)
    return step


def cpu_baseline(seconds=12.0):
    """The reference's CPU path (reference.py operations through the oracle port, torch.topk as
    the reference calls it) on the whole workload — all (batch, head) pairs — per step, on every
    host core: one warm-up step, then whole steps until ``seconds`` have passed (at least 2). The
    same computation as ``--impl reference``, so the two legs report one number."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    step = cpu_sample_step(WL["B"] * WL["H"])
    step()  # warm-up
    t0 = time.perf_counter()
    n = 0
    while True:
        step()
        n += 1
        if time.perf_counter() - t0 >= seconds and n >= 2:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": round(WL["B"] * WL["N"] / dt, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"the whole workload ({WL['B'] * WL['H']} of {WL['B'] * WL['H']} (batch,head) pairs) per "
                      f"step, fwd+bwd, fp32 CPU (reference.py operations, torch.topk); {n} timed steps of "
                      f"{dt * 1e3:.0f} ms after one warm-up step",
            "cpu": cpu_model()}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args):
    """The reference's CPU implementation of the path (the oracle port of reference.py, with
    torch.topk as the reference calls it) on all host cores, on the same workload as our arm:
    every step is one forward + backward over all (batch, head) pairs. Under torchrun only rank 0
    runs; the other ranks exit without work."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    pairs = WL["B"] * WL["H"]
    step = cpu_sample_step(pairs)
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    value = round(WL["B"] * WL["N"] / dt, 1)
    sample = (f"the whole workload ({pairs} of {pairs} (batch,head) pairs) per step, fwd+bwd, fp32 CPU "
              f"(reference.py operations, torch.topk)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": workload_config({"parallelism": "host CPU, one process"}),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample, "cpu": cpu_model()},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


LAYER = dict(B=2, N=8192, dim=1024, heads=16, slots=256, R=3)


def run_layer(args):
    """``--workload layer``: the layer training step alone (layer_leg) as the JSON line."""
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=dev)
    res = layer_leg(args, world, rank, dev, flush)
    if rank == 0:
        line = {"metric": "MurmurativeAttention layer training step tokens/s (BASELINE configs[3])",
                "value": res["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": res["workload"], "global_batch": res["global_batch"], "seq_len": res["seq_len"],
                           "parallelism": res["parallelism"], "l2": "flushed before every timed step by a kernel reading and writing 256 MiB"},
                "collective": {k: v for k, v in res.items() if k.startswith(("collective", "allreduce", "share"))}}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def surface_leg(args, dev, flush):
    """The reference's full op (ops.slot_murmurate, 6 arguments) on the north-star sizes:
    B=1, N=8192, 16 heads of d=64 (D=1024), M=256, R=3, fp16, separate q/k/v projections,
    residual x, a selection mask and a position bias; forward + backward through the
    per-phase CUDA-core kernels (murm_ops.cu)."""
    from murmurative_attention_b200 import functional as F
    B, N, H, Dh, M = 1, 8192, 16, 64, 256
    g = torch.Generator(device=dev).manual_seed(3000)
    mk = lambda *s, std=1.0: (torch.randn(*s, device=dev, generator=g) * std).half().requires_grad_(True)
    x, qp, kp, vp = (mk(B, N, H * Dh) for _ in range(4))
    ske, sve = mk(H, M, Dh), mk(H, M, Dh, std=0.5)
    mask = (torch.rand(N, M, device=dev, generator=g) > 0.1).to(torch.uint8)
    ramp = torch.linspace(-1.0, 1.0, M, device=dev, dtype=torch.float16)
    bias_fn = lambda xh: 0.1 * torch.tanh(xh[..., :1]) * ramp
    go = torch.randn(B, N, H * Dh, device=dev, generator=g).half()

    def step():
        out = F.slot_murmurate(x, qp, kp, vp, ske, sve, num_heads=H, rounds=3, mask=mask, position_bias_fn=bias_fn)
        out.backward(go)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ms = sum(time_steps(step, args.steps, flush)) / args.steps
    return {"metric": "ops.slot_murmurate (6-argument op surface) fwd+bwd tokens/s", "value": round(B * N / (ms / 1e3), 1),
            "unit": "tokens/s", "ms_per_step": round(ms, 5), "dtype": "fp16",
            "workload": "op surface: x, q/k/v projections [1,8192,1024], slot embeddings [16,256,64], "
                        "mask [8192,256] (90% kept), position bias from x, dynamic M, R=3",
            "path": "per-phase CUDA-core kernels (murm_ops.cu)"}


def decode_leg(args, dev, flush):
    """Streaming decode (the reference's decode plan): 16 sequences x 16 heads of d=64,
    M=256 resident slots, fp16, one token per sequence per step through murm_decode_step,
    the step replayed from a CUDA graph. tokens/s = sequences / step time."""
    from murmurative_attention_b200.decode import SlotPool
    B, H, M, D = 16, 16, 256, 64
    g = torch.Generator(device=dev).manual_seed(4000)
    ske = torch.randn(H, M, D, device=dev, generator=g).half()
    sve = (torch.randn(H, M, D, device=dev, generator=g) * 0.5).half()
    pool = SlotPool.from_embeddings(ske, sve, B)
    pool.positions.fill_(4096)
    q, k, v, x = (torch.randn(B, H * D, device=dev, generator=g).half() for _ in range(4))
    for _ in range(args.warmup):
        pool.step(q, k, v, x, causal=True)
    torch.cuda.synchronize()
    fn, graph = graph_of(lambda: pool.step(q, k, v, x, causal=True))
    ms = sum(time_steps(fn, args.steps, flush)) / args.steps
    return {"metric": "streaming decode tokens/s (one token per sequence per step)", "value": round(B / (ms / 1e3), 1),
            "unit": "tokens/s", "ms_per_step": round(ms, 5), "dtype": "fp16",
            "workload": "decode: 16 sequences x 16 heads, d=64, M=256 resident slots, causal, one launch per step",
            "pool_bytes_per_step": 2 * 2 * B * H * M * D * 2, "timing": "CUDA graph replay" if graph else "eager"}


def sp_leg(args, world, rank, dev, flush):
    """Sequence parallelism (sequence_parallel.slot_murmurate_sp) for a long context with few
    (batch, head) pairs: B=1, H=2, N=65536, d=64, M=256, R=3, fp16, causal; the tokens are split
    over the ranks (strong scaling), one NCCL all-reduce of the slot sums per round, and the
    slot gradients all-reduced after the backward. Forward + backward."""
    import torch.distributed as dist
    from murmurative_attention_b200.sequence_parallel import slot_murmurate_sp
    B, H, N, D, M = 1, 2, 65536, 64, 256
    n = N // world
    g = torch.Generator(device=dev).manual_seed(5000)
    q = torch.randn(B, H, N, D, device=dev, generator=g).half()[:, :, rank * n:(rank + 1) * n].contiguous()
    sk = torch.randn(B, H, M, D, device=dev, generator=g).half()
    sv = torch.zeros(B, H, M, D, device=dev, dtype=torch.float16)
    go = torch.randn(B, H, N, D, device=dev, generator=g).half()[:, :, rank * n:(rank + 1) * n].contiguous()
    qd, skd, svd = (t.clone().requires_grad_(True) for t in (q, sk, sv))

    def step():
        out, _, _ = slot_murmurate_sp(qd, skd, svd, rounds=3, causal=True)
        out.backward(go)
        if world > 1:
            dist.all_reduce(skd.grad)
            dist.all_reduce(svd.grad)
        qd.grad = skd.grad = svd.grad = None
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    times = time_steps(step, args.steps, flush)
    barrier(world)
    ms = max_over_ranks(sum(times), world) / args.steps
    return {"metric": "sequence-parallel slot_murmurate fwd+bwd (b,h)-tokens/s (long context, few (b,h))",
            "value": round(B * H * N / (ms / 1e3), 1), "unit": "(b,h)-tokens/s", "ms_per_step": round(ms, 5),
            "scaling": "strong", "dtype": "fp16",
            "workload": "sp: B=1, H=2, N=65536 split over the ranks, d=64, M=256, R=3, causal",
            "path": "per-phase kernels + one NCCL all-reduce of the slot sums per round", "parallelism": f"sp{world}"}


def _single(args, leg_name):
    """``--workload surface|decode|sp``: one leg alone as the JSON line."""
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=dev)
    if leg_name == "sp":
        res = sp_leg(args, world, rank, dev, flush)
    else:
        res = (surface_leg if leg_name == "surface" else decode_leg)(args, dev, flush)
    if rank == 0:
        line = {"metric": res.pop("metric"), "value": res.pop("value"), "unit": res.pop("unit"), "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": res.pop("ms_per_step"),
                "higher_is_better": True, "scaling": res.pop("scaling", "weak"), "vs_baseline": None,
                "dtype": res.pop("dtype"), "data": "synthetic", "config": res}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the cpu_baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--skip-strong", action="store_true", help="omit the configs[2] strong-scaling leg")
    ap.add_argument("--skip-layer", action="store_true", help="omit the configs[3] layer-step leg")
    ap.add_argument("--skip-widening", action="store_true",
                    help="omit the sequence-parallel, op-surface and decode legs")
    ap.add_argument("--dtype", choices=("fp16", "bf16"), default="fp16",
                    help="input dtype of the north-star workload (BASELINE configs[1] is fp16)")
    ap.add_argument("--workload", choices=("northstar", "layer", "surface", "decode", "sp"), default="northstar",
                    help="layer: BASELINE configs[3], the data-parallel layer training step; "
                         "surface: the reference's 6-argument op through the per-phase kernels; "
                         "decode: the streaming decode step; sp: sequence parallelism over the tokens")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    global DTYPE, DTYPE_NAME
    DTYPE, DTYPE_NAME = (torch.bfloat16, "bf16") if args.dtype == "bf16" else (torch.float16, "fp16")
    if args.workload != "northstar":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": f"the {args.workload} workload has no reference arm here"}))
            return
        if args.workload == "layer":
            run_layer(args)
        else:
            _single(args, args.workload)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
