"""Gated DeltaNet forward + backward tokens/s on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c1|c2|c3|c4|conv_norm]

One step is the whole training pass of the recurrence's layer slice over one batch, through the fused
layer entry points (the norm and gate graph inside the chunked kernels):
    layer forward (raw q, k normalised; log g, beta from a, b, A_log, dt_bias; y, final state, chunk
    intermediates saved) -> layer backward (dq, dk through the norms, dv, da, db, per-head dA_log,
    ddt_bias given dy) -> when the batch is split over GPUs, one all-reduce of [dA_log | ddt_bias] (NCCL).
With --algo 1 the row-parallel kernels run instead, with the gate graph as separate kernels.

Workloads (synthetic, seeded; shapes and value distributions of the measured configurations):
  c1  Qwen3.5-4B layer: B=1 per GPU, T=2048, Hk=16, Hv=32, Dk=Dv=128, bf16 activations, fp32 g/beta/state.
      Weak scaling: GPU r runs batch row r (global batch = N).
  c2  B=8, T=4096, Hk=16, Hv=64 split over the GPUs by (batch x value-head group); strong scaling.
  c3  16 sequences of U[128, 4096] tokens packed with cu_seqlens (one GPU); sub-result: one sequence of
      T=32768 with an initial state and a final-state gradient.
  c4  exact speculative verify of 8 drafted tokens for 32 sequences, every state kept (one GPU);
      sub-result: the decode-time companions (the conv's verify rows, keep_conv_rows, keep_rows).
  conv_norm  the layer's steps either side of the recurrence at the 4B shape, 4 x 2048 tokens: the causal
      conv + SiLU with the q/k/v split and the gated RMSNorm, forward and backward (one GPU; HBM-bound).

`value` is tokens/s of the whole job (tokens of all ranks / max over ranks of the device time);
`e2e` is the same metric through the public API with host buffers: every step copies its inputs
from pinned host memory (packed in one buffer, one copy) and its gradients back.  L2 is flushed (a
512 MiB write) before each timed step and the flush is outside the step's events.  With N ranks the
GPUs are aligned before the timed steps (an all-reduce, then a short device sleep while every host
enqueues), so that no rank's events include waiting for a peer whose process started late.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CHUNK = 64


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c1", choices=["c1", "c2", "c3", "c4", "conv_norm"],
                    help="c1 4B layer (default), c2 batched split over GPUs, c3 varlen (one GPU), c4 verify (one GPU), "
                         "conv_norm the conv and gated norm around the recurrence (one GPU)")
    ap.add_argument("--algo", type=int, default=0, help="0 auto, 1 row-parallel, 2 chunked")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-c2", action="store_true", help="skip the config 2 strong-scaling sub-result")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="time eager launches instead of a CUDA graph of the step")
    return ap.parse_args()


# ---- algorithmic work (chunk C = 64, dense contractions only; bytes read once, written once) ----
def fwd_flops_per_token_head(Dk, Dv, C=CHUNK):
    return (2 * C * C * (3 * Dk + 2 * Dv) + 6 * C * Dk * Dv + (2.0 / 3.0) * C ** 3) / C


def bytes_per_token(Hk, Hv, Dk, Dv, act=2):
    fwd = 2 * Hk * Dk * act + Hv * Dv * act + 2 * Hv * 4 + Hv * Dv * act
    bwd = (2 * Hk * Dk * act + 2 * Hv * Dv * act + 2 * Hv * 4) + (2 * Hk * Dk * act + Hv * Dv * act + 2 * Hv * 4)
    return fwd, bwd


# DRAM bytes (read + write) per launch of the dominant op, copied from one ncu capture of this bench's
# workload (dram__bytes_read.sum + dram__bytes_write.sum); a constant, so it goes stale when the kernels
# change and is refreshed from a new capture then.  None where no capture was made.
TRAFFIC = {("c1", "layer_bwd"): 456.0e6, ("c4", "verify"): 550.8e6}
TRAFFIC_NOTE = "constant from one ncu capture of this workload (not measured in this run)"


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ---- clocks during the timed region ----
class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region.  NVML is polled back to back (the
    timed region of one workload is milliseconds to tens of milliseconds, too short for nvidia-smi's 200 ms
    period); nvidia-smi -lms 200 is the fallback when NVML cannot be loaded."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.thread = None
        self.lines = []
        self.sm = []
        self.reasons = set()
        self.max_mhz = None
        self.source = None
        self.n_reason_polls = 0
        self._stop = threading.Event()

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            bits = {"hw_slowdown": pynvml.nvmlClocksThrottleReasonHwSlowdown,
                    "hw_thermal_slowdown": getattr(pynvml, "nvmlClocksThrottleReasonHwThermalSlowdown", 0x40),
                    "sw_thermal_slowdown": getattr(pynvml, "nvmlClocksThrottleReasonSwThermalSlowdown", 0x20),
                    "sw_power_cap": pynvml.nvmlClocksThrottleReasonSwPowerCap}

            def poll():  # the SM clock every poll, the throttle reasons every fourth (and on the last)
                k = 0
                while True:
                    last = self._stop.is_set()
                    try:
                        self.sm.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                        if k % 4 == 0 or last:
                            r = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                            self.n_reason_polls += 1
                            for n, b in bits.items():
                                if r & b:
                                    self.reasons.add(n)
                    except Exception:
                        pass
                    if last:
                        break
                    k += 1
                    time.sleep(0.0001)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            self.source = "nvml: SM clock polled back to back, throttle reasons every fourth poll"
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            self.source = "nvidia-smi -lms 200"
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            for line in self.lines:
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    self.sm.append(float(f[1]))
                    self.max_mhz = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(self.NAMES, f[5:9]):
                    if v.lower() == "active":
                        self.reasons.add(n)
        elif self.thread is not None:
            self.thread.join(timeout=1)
        if self.source is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"]}
        sm = sorted(self.sm)
        med = sm[len(sm) // 2] if sm else None
        out = {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(sm),
               "source": self.source}
        if self.n_reason_polls:
            out["reason_samples"] = self.n_reason_polls
        return out


# ---- the step ----
class Work:
    """One rank's share of the workload, resident in HBM."""

    def __init__(self, B, T, Hk, Hv, Dk, Dv, seed, device, algo, cu_seqlens=None, with_state=False):
        from quotebound_b200 import synthetic
        p = synthetic.make(B, T, Hk, Hv, Dk, Dv, seed=seed, device=device)
        self.cu = cu_seqlens
        gen = torch.Generator(device=device).manual_seed(seed + 7)
        # raw (pre-norm) q, k: any positive rescale of the normalised vectors gives the same qn, kn
        self.q = (p.q * math.sqrt(Dk) * torch.rand(B, T, Hk, 1, generator=gen, device=device).add_(0.5)).to(torch.bfloat16)
        self.k = (p.k * torch.rand(B, T, Hk, 1, generator=gen, device=device).add_(0.5)).to(torch.bfloat16)
        self.v = p.v.to(torch.bfloat16)
        self.a, self.b = p.a.contiguous(), p.b.contiguous()
        self.A_log, self.dt_bias = p.A_log, p.dt_bias
        self.dy = p.dy.to(torch.bfloat16)
        self.shape = (B, T, Hk, Hv, Dk, Dv)
        self.algo = algo
        # an initial state and a final-state gradient, both ~ N(0, 0.02) (config 3's long sequence)
        self.h0 = self.dhT = None
        if with_state:
            self.h0 = torch.randn(B, Hv, Dv, Dk, generator=gen, device=device) * 0.02
            self.dhT = torch.randn(B, Hv, Dv, Dk, generator=gen, device=device) * 0.02

    def step(self, events=None):
        """One fwd+bwd pass; returns (grads..., dA_log, ddt_bias).  `events`: list to append (name, ev0, ev1)."""
        from quotebound_b200 import deltanet, gate

        def op(name, fn):
            if events is None:
                return fn()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn()
            e1.record()
            events.append((name, e0, e1))
            return out

        cu = getattr(self, "cu", None)
        if self.algo != 1:  # the fused layer path: norm, gates and recurrence in the chunked kernels
            from quotebound_b200 import layer
            h0, dhT = getattr(self, "h0", None), getattr(self, "dhT", None)
            y, hT, saved = op("layer_fwd", lambda: layer.gated_delta_layer_fwd(
                self.q, self.k, self.v, self.a, self.b, self.A_log, self.dt_bias, h0, save=True, cu_seqlens=cu))
            dq, dk, dv, da, db, dA, ddt, _ = op("layer_bwd", lambda: layer.gated_delta_layer_bwd(
                self.q, self.k, self.v, self.a, self.b, self.A_log, self.dt_bias, h0, self.dy, dhT, saved=saved,
                cu_seqlens=cu))
            return dq, dk, dv, da, db, dA, ddt
        qn, kn, g, beta = op("gate_fwd", lambda: gate.gate_fwd(self.q, self.k, self.a, self.b, self.A_log,
                                                                 self.dt_bias))
        y, hT, saved = op("gdn_fwd", lambda: deltanet.gated_delta_fwd(qn, kn, self.v, g, beta, None, save=True,
                                                                       algo=self.algo, cu_seqlens=cu))
        dqn, dkn, dv, dg, dbeta, _ = op("gdn_bwd", lambda: deltanet.gated_delta_bwd(
            qn, kn, self.v, g, beta, None, self.dy, None, saved=saved, algo=self.algo, cu_seqlens=cu))
        dq, dk, da, db, dA, ddt = op("gate_bwd", lambda: gate.gate_bwd(self.q, self.k, self.a, self.b, self.A_log,
                                                                        self.dt_bias, dqn, dkn, dg, dbeta))
        return dq, dk, dv, da, db, dA, ddt


def rank_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def workload_shape(name, world, rank):
    """(B, T, Hk, Hv, Dk, Dv, seed, tokens of this rank, description)."""
    if name == "c1":
        return 1, 2048, 16, 32, 128, 128, rank, 2048
    from quotebound_b200 import partition
    shards = partition.plan(B=8, Hk=16, Hv=64, world=world)
    s = shards[rank]
    nb, nhk = s.b1 - s.b0, s.hk1 - s.hk0
    return nb, 4096, nhk, nhk * 4, 128, 128, 1000 + rank, nb * 4096 * nhk * 4 / 64  # tokens weighted by heads


def flush_l2(buf):
    buf.zero_()


def _measure(args, workload, world, rank, dev, dist, steps, warmup):
    """One workload on this rank: the step captured in a CUDA graph, W warm-up then K timed steps (L2
    flushed before each, outside its events), the per-op split from eager steps.  Returns a dict."""
    from quotebound_b200 import _lib, partition
    B, T, Hk, Hv, Dk, Dv, seed, _ = workload_shape(workload, world, rank)
    W = Work(B, T, Hk, Hv, Dk, Dv, seed, dev, args.algo)
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)
    Hv_all = 64 if workload == "c2" else Hv
    red = torch.empty(2 * Hv_all, dtype=torch.float32, device=dev)
    shard = partition.plan(B=8, Hk=16, Hv=64, world=world)[rank] if workload == "c2" else None
    reduces = dist and (workload == "c1" or partition.needs_allreduce(partition.plan(B=8, Hk=16, Hv=64, world=world)))

    def allreduce(dA, ddt):
        if not reduces:
            return
        if shard is not None:
            red.zero_()
            red[shard.hv0:shard.hv1] = dA
            red[64 + shard.hv0:64 + shard.hv1] = ddt
        else:
            red[:Hv] = dA
            red[Hv:] = ddt
        torch.distributed.all_reduce(red)

    for _ in range(warmup):
        out = W.step()
        allreduce(out[5], out[6])
    torch.cuda.synchronize()

    # The step's launches captured once in a CUDA graph and replayed (the library's host-side work --
    # argument checks, tensor maps, workspace allocation -- then costs nothing per step).  With several
    # ranks the all-reduce is captured too (NCCL supports capture; the communicator was created by the
    # eager warm-up); if that capture fails, the graph holds the step alone and the all-reduce runs eagerly.
    graph, gout, graph_launches, graph_reduces = None, None, 0, False
    if not args.no_graph:
        for with_reduce in ((True, False) if reduces else (False,)):
            try:
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    W.step()
                torch.cuda.current_stream().wait_stream(side)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                n_cap = _lib.launches()
                with torch.cuda.graph(graph):
                    gout = W.step()
                    if with_reduce:
                        allreduce(gout[5], gout[6])
                graph_launches = _lib.launches() - n_cap
                graph.replay()
                torch.cuda.synchronize()
                graph_reduces = with_reduce
                break
            except Exception as exc:  # capture unsupported here: try without the collective, then eager
                print(f"bench: CUDA graph capture failed ({exc})", file=sys.stderr)
                graph, gout = None, None
                torch.cuda.synchronize()

    sampler = ClockSampler(dev.index)
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    if dist:
        # The ranks' processes leave the barrier at different moments; a GPU whose timed steps start early
        # would wait inside its first step's all-reduce for a peer whose host started late, and that wait
        # would count in its events.  So the GPUs are aligned first: an all-reduce that all of them leave
        # together, then a device sleep of about 20 ms during which every host enqueues its timed steps.
        align = torch.zeros(1, device=dev)
        torch.distributed.all_reduce(align)
        torch.cuda._sleep(40_000_000)
    sampler.start()
    n0 = _lib.launches()
    step_events, op_events = [], []
    for _ in range(steps):
        flush_l2(flush)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        if graph is not None:
            graph.replay()
            if not graph_reduces:
                allreduce(gout[5], gout[6])
        else:
            out = W.step(op_events)
            allreduce(out[5], out[6])
        e1.record()
        step_events.append((e0, e1))
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
    launches = (_lib.launches() - n0) + graph_launches * steps
    clocks = sampler.stop()
    ms = sum(a.elapsed_time(b) for a, b in step_events) / steps
    if graph is not None:  # the per-op split from eager steps (after eager warm-up: the graph's pool is its own)
        for k in range(3 + steps):
            flush_l2(flush)
            out = W.step(op_events if k >= 3 else None)
            allreduce(out[5], out[6])
        torch.cuda.synchronize()
    per_op = {}
    for name, a, b in op_events:
        per_op.setdefault(name, []).append(a.elapsed_time(b))
    per_op = {k: sum(v) / len(v) for k, v in per_op.items()}
    ms_max, ms_ranks = ms, [round(ms, 4)]
    if dist:
        t = torch.zeros(world, device=dev)
        t[rank] = ms
        torch.distributed.all_reduce(t)  # every rank's time (the others contribute zeros)
        ms_ranks = [round(float(x), 4) for x in t.tolist()]
        ms_max = max(ms_ranks)
    total_tokens = world * B * T if workload == "c1" else 8 * 4096
    return {"W": W, "allreduce": allreduce, "graph": graph, "gout": gout, "graph_reduces": graph_reduces,
            "ms_max": ms_max, "ms_ranks": ms_ranks, "per_op": per_op, "launches": launches, "clocks": clocks, "B": B, "T": T, "Hk": Hk,
            "Hv": Hv, "Dk": Dk, "Dv": Dv, "value": total_tokens / (ms_max / 1e3), "reduces": reduces,
            "flush": flush}


def _roofline(workload, per_op, B, T, Hk, Hv, Dk, Dv):
    hbm, tf, src = load_peaks()
    fpt = fwd_flops_per_token_head(Dk, Dv)
    dom = max(per_op, key=per_op.get)  # the dominant op of the step and its algorithmic work per launch
    toks = B * T
    flops = {"gdn_fwd": fpt * toks * Hv, "gdn_bwd": 2 * fpt * toks * Hv, "layer_fwd": fpt * toks * Hv,
             "layer_bwd": 2 * fpt * toks * Hv}
    fb, bb = bytes_per_token(Hk, Hv, Dk, Dv)
    bytes_ = {"gdn_fwd": fb * toks, "gdn_bwd": bb * toks, "layer_fwd": fb * toks, "layer_bwd": bb * toks,
              "gate_fwd": toks * (2 * Hk * Dk * 2 * 2 + Hv * 4 * 4),
              "gate_bwd": toks * (4 * Hk * Dk * 2 + 2 * Hk * Dk * 2 + Hv * 4 * 6)}
    dom_ms = per_op[dom]
    if dom in flops:
        ach = flops[dom] / (dom_ms / 1e3) / 1e12
        return {"kernel": dom, "bound": "tensor", "achieved": round(ach, 3), "peak": tf, "unit": "TFLOP/s",
                "frac": round(ach / tf, 5), "peak_source": src, "traffic": TRAFFIC.get((workload, dom)),
                "traffic_source": TRAFFIC_NOTE, "ms_per_launch": round(dom_ms, 4),
                "flop_per_launch": flops[dom], "bytes_per_launch": bytes_[dom],
                "hbm_achieved_gbs": round(bytes_[dom] / (dom_ms / 1e3) / 1e9, 1),
                "hbm_frac": round(bytes_[dom] / (dom_ms / 1e3) / 1e9 / hbm, 5)}
    ach = bytes_[dom] / (dom_ms / 1e3) / 1e9
    return {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(ach / hbm, 5), "peak_source": src, "traffic": TRAFFIC.get((workload, dom)),
            "traffic_source": TRAFFIC_NOTE, "ms_per_launch": round(dom_ms, 4)}


def run_ours(args):
    world, rank, local = rank_info()
    dist = world > 1
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if dist:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    from quotebound_b200 import _lib, build
    build.ensure()
    _lib.load()
    m = _measure(args, args.workload, world, rank, dev, dist, args.steps, args.warmup)
    # e2e through the public API with host buffers (pinned), every step: H2D inputs, D2H gradients
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(m["W"], args, dev, dist, world, m["allreduce"])
    graph = m.pop("graph")
    m.pop("gout")
    # config 2 beside config 1: B=8, T=4096, Hv=64 split by (batch x head group) over the same ranks,
    # fixed total work (strong scaling) -- the curve that exercises the partitioner and its all-reduce
    c2 = None
    if args.workload == "c1" and not args.no_c2:
        del graph
        torch.cuda.synchronize()
        n2 = _measure(args, "c2", world, rank, dev, dist, max(3, args.steps // 2), max(3, args.warmup))
        n2.pop("graph"), n2.pop("gout")
        c2 = n2
        graph = None

    if rank == 0:
        workload = args.workload
        line = {
            "metric": "GDN fwd+bwd tokens/s at 4B layer shape" if workload == "c1"
            else "GDN fwd+bwd tokens/s, B=8 T=4096 Hv=64 split over GPUs",
            "value": round(m["value"], 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(m["ms_max"], 4), "ms_per_rank": m["ms_ranks"],
            "higher_is_better": True,
            "scaling": "weak" if workload == "c1" else "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; q,k,v,dO ~ N(0,1), q/k normalised, g = exp(-e^A_log softplus(a+dt_bias)))",
            "config": {"workload": "config1: B=1/GPU T=2048 Hk=16 Hv=32 Dk=Dv=128" if workload == "c1"
                       else "config2: B=8 T=4096 Hk=16 Hv=64 Dk=Dv=128, (batch x head-group) split",
                       "global_batch": world * m["B"] if workload == "c1" else 8, "seq_len": m["T"],
                       "parallelism": f"dp{world}" if workload == "c1" else f"bh{world}",
                       "l2": "flushed before every step (512 MiB write, outside the step events)",
                       "ranks": "aligned before the timed steps (an all-reduce, then a device sleep while every "
                                "host enqueues); the line's time is the slowest rank's" if world > 1 else "one",
                       "launch": "CUDA graph of the step" + (" and its all-reduce" if m["graph_reduces"] else "")
                       + ", replayed",
                       "algo": {0: "auto", 1: "rows", 2: "chunked"}[args.algo],
                       "step": ("layer_fwd(save) + layer_bwd" if args.algo != 1 else
                                "gate_fwd + gdn_fwd(save) + gdn_bwd + gate_bwd")
                       + (" + allreduce" if m["reduces"] else "")},
            "per_op_ms": {k: round(v, 4) for k, v in m["per_op"].items()},
            "gpu_launches": int(m["launches"]),
            "clocks": m["clocks"],
            "roofline": _roofline(workload, m["per_op"], m["B"], m["T"], m["Hk"], m["Hv"], m["Dk"], m["Dv"]),
            "e2e": e2e,
        }
        if c2 is not None:
            line["config2_strong"] = {
                "metric": "GDN fwd+bwd tokens/s, config2 (B=8 T=4096 Hk=16 Hv=64) split over the GPUs",
                "value": round(c2["value"], 1), "unit": "tokens/s", "n_gpus": world, "scaling": "strong",
                "ms_per_step": round(c2["ms_max"], 4), "ms_per_rank": c2["ms_ranks"], "steps": max(3, args.steps // 2),
                "per_rank": {"batch_rows": c2["B"], "key_heads": c2["Hk"], "value_heads": c2["Hv"]},
                "allreduce": c2["reduces"], "per_op_ms": {k: round(v, 4) for k, v in c2["per_op"].items()},
                "gpu_launches": int(c2["launches"]), "clocks": c2["clocks"],
                "roofline": _roofline("c2", c2["per_op"], c2["B"], c2["T"], c2["Hk"], c2["Hv"], c2["Dk"], c2["Dv"])}
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(workload)
        print(json.dumps(line), flush=True)
    # a graph that holds an NCCL call is released before its process group
    del graph
    m.clear()
    if c2 is not None:
        c2.clear()
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_e2e(W, args, dev, dist, world, allreduce):
    """Same step through the public API with host buffers, as a training input pipeline runs it: every
    step's inputs go host-to-device from pinned memory on a copy stream (overlapping the previous step's
    compute, double-buffered on the device), and every gradient comes back device-to-host on a second
    stream (overlapping the next step's compute).  The timed region spans all of it: the first step's
    upload to the last step's download."""
    names = ("q", "k", "v", "a", "b", "dy")
    # a step's inputs packed in one pinned buffer (256-byte aligned slots), uploaded by one copy into one
    # of two device buffers whose slots are the tensors the step reads
    offs, total = {}, 0
    for n in names:
        t = getattr(W, n)
        offs[n] = total
        total += (t.numel() * t.element_size() + 255) // 256 * 256
    host_buf = torch.empty(total, dtype=torch.uint8).pin_memory()
    dev_buf = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(2)]

    def slot(buf, n):
        t = getattr(W, n)
        return buf[offs[n]:offs[n] + t.numel() * t.element_size()].view(t.dtype).view(t.shape)

    for n in names:
        slot(host_buf, n).copy_(getattr(W, n).cpu())
    dev_in = [{n: slot(dev_buf[i], n) for n in names} for i in range(2)]
    outs = W.step()
    host_out = [o.cpu().pin_memory() for o in outs]
    h2d = total  # the bytes the copy moves (the inputs and their slots' padding)
    d2h = sum(t.numel() * t.element_size() for t in host_out)

    class HostWork:
        pass

    hws = []
    for i in range(2):
        hw = HostWork()
        for n in ("A_log", "dt_bias", "shape", "algo"):
            setattr(hw, n, getattr(W, n))
        for n, t in dev_in[i].items():
            setattr(hw, n, t)
        hws.append(hw)
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    loaded = [torch.cuda.Event() for _ in range(2)]   # set i holds its step's inputs
    freed = [torch.cuda.Event() for _ in range(2)]    # the step that read set i has finished
    freed_used = [False, False]

    def upload(i):
        if freed_used[i]:
            s_in.wait_event(freed[i])
        with torch.cuda.stream(s_in):
            dev_buf[i].copy_(host_buf, non_blocking=True)
            loaded[i].record(s_in)

    def compute(i):
        comp.wait_event(loaded[i])
        out = Work.step(hws[i])
        allreduce(out[5], out[6])
        freed[i].record(comp)
        freed_used[i] = True
        s_out.wait_event(freed[i])
        with torch.cuda.stream(s_out):
            for h, o in zip(host_out, out):
                h.copy_(o, non_blocking=True)
                o.record_stream(s_out)

    def run(nsteps, start):
        s_in.wait_event(start)
        upload(0)
        for k in range(nsteps):
            if k + 1 < nsteps:
                upload((k + 1) % 2)
            compute(k % 2)
        fin = torch.cuda.Event()
        fin.record(s_out)
        comp.wait_event(fin)

    w0 = torch.cuda.Event()
    w0.record(comp)
    run(max(2, args.warmup), w0)
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    n = max(3, args.steps)  # K steps, as the device-timed line; the pipeline's fill and drain included
    run(n, e0)
    e1.record(comp)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    if dist:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    B, T = W.shape[0], W.shape[1]
    total = (world * B * T) if args.workload == "c1" else 8 * 4096
    return {"value": round(total / (ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": round(ms, 4), "steps": n,
            "pipeline": "H2D of step k+1 (the inputs packed in one pinned buffer, one copy) and D2H of step k-1 "
                        "overlap step k's compute (separate streams)"}


# ---- the CPU side: the oracle on the host cores ----
def _oracle_sample(T, threads, seconds):
    """Times the CPU oracle's fwd+bwd on config 1's heads over T steps until `seconds` have passed."""
    from oracle import oracle
    import numpy as np
    from quotebound_b200 import synthetic
    p = synthetic.make(1, T, 16, 32, 128, 128, seed=0)
    q = p.q.to(torch.bfloat16).float().numpy()
    k = p.k.to(torch.bfloat16).float().numpy()
    v = p.v.to(torch.bfloat16).float().numpy()
    dy = p.dy.to(torch.bfloat16).float().numpy()
    g, beta = p.g.numpy(), p.beta.numpy()
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.gated_delta_fwd(q, k, v, g, beta, None, acc64=False, threads=threads)
        oracle.gated_delta_bwd(q, k, v, g, beta, None, dy, None, acc64=False, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return n * T / el, n, el


def cpu_baseline(workload):
    """The CPU oracle on every host core over config 1 itself (T=2048), about ten seconds of passes."""
    from oracle import oracle
    oracle.build()
    threads = os.cpu_count() or 1
    T = 2048
    tps, n, el = _oracle_sample(T, threads, 10.0)
    return {"value": round(tps, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"config1 (B=1, T={T}, Hk=16, Hv=32, Dk=Dv=128) fwd+bwd, float32 C oracle, OpenMP "
                      f"{threads} threads, {n} passes in {el:.1f} s"}


def run_reference(args):
    """The reference's CPU path for this recurrence (its MLX/Metal build cannot run here): the C oracle
    restating it, on every host core, on config 1 itself (B=1, T=2048, Hk=16, Hv=32, Dk=Dv=128): each
    step is one forward + backward pass over the whole sequence."""
    world, rank, local = rank_info()
    if rank != 0:
        return
    from oracle import oracle
    oracle.build()
    threads = os.cpu_count() or 1
    T = 2048
    for _ in range(args.warmup):
        _oracle_sample(T, threads, 0.0)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        _oracle_sample(T, threads, 0.0)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    v = T / (ms / 1e3)
    line = {"impl": "reference", "metric": "GDN fwd+bwd tokens/s at 4B layer shape", "value": round(v, 1),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "dtype": "f32",
            "config": {"workload": "config1: B=1 T=2048 Hk=16 Hv=32 Dk=Dv=128", "same_config": True},
            "cpu_baseline": {"value": round(v, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"one fwd+bwd of config 1 (T={T}) per timed step, mean of {args.steps}"},
            "e2e": {"value": round(v, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's recurrence runs on MLX/Metal (macOS only); its CPU restatement is timed"}
    print(json.dumps(line), flush=True)


# ---- one-GPU workloads: config 3 (varlen training pass) and config 4 (exact speculative verify) ----
def _timed(step, steps, warmup, dev):
    """Mean device ms of `step(events)` over `steps` (L2 flushed before each, outside the events)."""
    from quotebound_b200 import _lib
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for _ in range(warmup):
        step(None)
    torch.cuda.synchronize()
    sampler = ClockSampler(dev.index)
    sampler.start()
    n0 = _lib.launches()
    evs, ops = [], []
    for _ in range(steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        step(ops)
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    launches = _lib.launches() - n0
    clocks = sampler.stop()
    ms = sum(a.elapsed_time(b) for a, b in evs) / steps
    per_op = {}
    for name, a, b in ops:
        per_op.setdefault(name, []).append(a.elapsed_time(b))
    return ms, {k: sum(v) / len(v) for k, v in per_op.items()}, launches, clocks


def _graph_ops_timed(ops, steps, warmup, dev, flush_bytes=256 * 1024 * 1024):
    """Each (name, fn) of `ops` captured in its own CUDA graph (its host-side work -- argument checks, output
    and workspace allocation, the ctypes call -- then stays out of its events) and replayed `steps` times,
    L2 flushed before each replay, outside its events, so that each op's inputs come from HBM.  Returns the
    mean device ms per op, the library launches in the timed replays and the clock record."""
    from quotebound_b200 import _lib
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device=dev)
    for _ in range(warmup):
        for _, fn in ops:
            fn()
    torch.cuda.synchronize()
    graphs = []
    for name, fn in ops:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        n_cap = _lib.launches()
        with torch.cuda.graph(g):
            fn()
        graphs.append((name, g, _lib.launches() - n_cap))
        g.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(dev.index)
    sampler.start()
    evs = []
    for _ in range(steps):
        for name, g, _ in graphs:
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            evs.append((name, e0, e1))
    torch.cuda.synchronize()
    clocks = sampler.stop()
    launches = sum(n for _, _, n in graphs) * steps
    per_op = {}
    for name, a, b in evs:
        per_op.setdefault(name, []).append(a.elapsed_time(b))
    return {k: sum(v) / len(v) for k, v in per_op.items()}, launches, clocks


def conv_norm_line(args, dev, hbm, src):
    """The causal conv + SiLU (with the q/k/v split) and the gated RMSNorm, forward and backward, at the 4B
    layer shape (Hk=16, Hv=32, Dk=Dv=128, conv_dim 8192, 4 taps) over B = 4 sequences of 2048 tokens: every
    activation is 64-128 MB, so each op streams HBM.  The roofline is each op's algorithmic bytes (its
    inputs read and outputs written once) over its CUDA-event time."""
    from quotebound_b200 import conv, norm
    B, T, Hk, Hv, D, K = 4, 2048, 16, 32, 128, 4
    cdim = 2 * Hk * D + Hv * D
    gen = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(B, T, cdim, generator=gen, device=dev).to(torch.bfloat16)
    w = (torch.randn(cdim, K, generator=gen, device=dev) * 0.5).to(torch.bfloat16)
    st = torch.randn(B, K - 1, cdim, generator=gen, device=dev).to(torch.bfloat16)
    dq = torch.randn(B, T, Hk, D, generator=gen, device=dev).to(torch.bfloat16)
    dk = torch.randn(B, T, Hk, D, generator=gen, device=dev).to(torch.bfloat16)
    dv = torch.randn(B, T, Hv, D, generator=gen, device=dev).to(torch.bfloat16)
    y = torch.randn(B, T, Hv, D, generator=gen, device=dev).to(torch.bfloat16)
    z = torch.randn(B, T, Hv, D, generator=gen, device=dev).to(torch.bfloat16)
    do = torch.randn(B, T, Hv, D, generator=gen, device=dev).to(torch.bfloat16)
    nw = torch.rand(D, generator=gen, device=dev) + 0.5

    ops = (("conv_fwd", lambda: conv.conv_fwd(x, w, st, Hk=Hk, Dk=D, Hv=Hv, Dv=D)),
           ("conv_bwd", lambda: conv.conv_bwd(x, w, st, dq, dk, dv, Hk=Hk, Dk=D, Hv=Hv, Dv=D)),
           ("norm_fwd", lambda: norm.gated_norm_fwd(y, z, nw)),
           ("norm_bwd", lambda: norm.gated_norm_bwd(y, z, nw, do)))
    per_op, launches, clocks = _graph_ops_timed(ops, args.steps, args.warmup, dev)
    ms = sum(per_op.values())  # the four ops' device time per step (the flushes between them excluded)
    act, row = B * T * cdim * 2, B * T * Hv * D * 2
    nbytes = {"conv_fwd": 2 * act, "conv_bwd": 3 * act, "norm_fwd": 3 * row, "norm_bwd": 5 * row}
    roof = {k: {"achieved_gbs": round(nbytes[k] / (per_op[k] / 1e3) / 1e9, 1),
                "frac": round(nbytes[k] / (per_op[k] / 1e3) / 1e9 / hbm, 4), "bytes": nbytes[k]} for k in nbytes}
    dom = max(per_op, key=per_op.get)
    return {"metric": "GDN layer conv + gated norm fwd+bwd tokens/s", "value": round(B * T / (ms / 1e3), 1),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded)",
            "config": {"workload": f"conv_norm: B={B} T={T} Hk={Hk} Hv={Hv} Dk=Dv={D} conv_dim={cdim} taps={K}",
                       "l2": "flushed before every op",
                       "step": "conv_fwd + conv_bwd + gated_norm_fwd + gated_norm_bwd, each a CUDA graph replay "
                               "(sum of the ops' event times)"},
            "per_op_ms": {k: round(v, 4) for k, v in per_op.items()}, "gpu_launches": int(launches),
            "clocks": clocks,
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": roof[dom]["achieved_gbs"], "peak": hbm,
                         "unit": "GB/s", "frac": roof[dom]["frac"], "peak_source": src, "traffic": None,
                         "bytes_per_launch": nbytes[dom], "per_op": roof}}


def decode_line(args, dev, hbm, N, V, Hk, Hv, D, rstates):
    """The decode-time companions of the verify at config 4's shape: the conv's verify rows (V drafted
    tokens of x through the conv + SiLU as V one-token steps, every token's conv window kept) and the two
    selections after acceptance (keep_conv_rows, keep_rows: the states after keep[n] accepted tokens).
    Each op a CUDA graph replay after an L2 flush; the roofline is each op's algorithmic bytes."""
    from quotebound_b200 import conv, exact
    K = 4
    cdim = 2 * Hk * D + Hv * D
    gen = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(N, V, cdim, generator=gen, device=dev).to(torch.bfloat16)
    w = (torch.randn(cdim, K, generator=gen, device=dev) * 0.5).to(torch.bfloat16)
    st = torch.randn(N, K - 1, cdim, generator=gen, device=dev).to(torch.bfloat16)
    cstates = conv.conv_verify(x, w, st, Hk=Hk, Dk=D, Hv=Hv, Dv=D)[3]
    keep = torch.randint(1, V + 1, (N,), generator=gen, device=dev, dtype=torch.int32)
    ops = (("conv_verify", lambda: conv.conv_verify(x, w, st, Hk=Hk, Dk=D, Hv=Hv, Dv=D)),
           ("keep_conv_rows", lambda: conv.keep_conv_rows(cstates, keep)),
           ("keep_rows", lambda: exact.keep_rows(rstates, keep)))
    per_op, launches, clocks = _graph_ops_timed(ops, args.steps, args.warmup, dev)
    nbytes = {"conv_verify": 2 * (2 * N * V * cdim + N * (K - 1) * cdim + N * V * (K - 1) * cdim) + cdim * K * 2,
              "keep_conv_rows": 2 * 2 * N * (K - 1) * cdim,
              "keep_rows": 2 * 4 * N * Hv * D * D}
    return {"config": f"N={N} sequences x V={V} drafted tokens, conv_dim {cdim}, K={K} taps, Hv={Hv}, Dv=Dk={D}",
            "per_op_ms": {k: round(v, 4) for k, v in per_op.items()},
            "roofline": {k: {"achieved_gbs": round(nbytes[k] / (per_op[k] / 1e3) / 1e9, 1),
                             "frac": round(nbytes[k] / (per_op[k] / 1e3) / 1e9 / hbm, 4), "bytes": nbytes[k]}
                         for k in nbytes},
            "gpu_launches": int(launches), "clocks": clocks,
            "timing": "each op a CUDA graph replay after an L2 flush (256 MiB write, outside its events)"}


def run_single(args):
    world, rank, local = rank_info()
    if world > 1:
        raise SystemExit("workloads c3, c4 and conv_norm run on one GPU")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from quotebound_b200 import _lib, build, exact, synthetic
    build.ensure()
    _lib.load()
    hbm, tf, src = load_peaks()
    if args.workload == "c3":
        lengths = synthetic.varlen_lengths(16, 128, 4096, seed=0)
        cu = synthetic.cu_from_lengths(lengths)
        T = cu[-1]
        W = Work(1, T, 16, 32, 128, 128, 0, dev, args.algo, cu_seqlens=cu)
        ms, per_op, launches, clocks = _timed(W.step, args.steps, args.warmup, dev)
        fpt = fwd_flops_per_token_head(128, 128)
        dom = "layer_bwd" if "layer_bwd" in per_op else "gdn_bwd"
        dom_ms = per_op[dom]
        ach = 2 * fpt * T * 32 / (dom_ms / 1e3) / 1e12
        line = {"metric": "GDN fwd+bwd tokens/s, varlen packed batch", "value": round(T / (ms / 1e3), 1),
                "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded)",
                "config": {"workload": f"config3: 16 sequences, lengths U[128,4096] (seed 0), {T} tokens, "
                                       "Hk=16 Hv=32 Dk=Dv=128, cu_seqlens",
                           "l2": "flushed before every step", "step": "layer_fwd(save) + layer_bwd"},
                "per_op_ms": {k: round(v, 4) for k, v in per_op.items()}, "gpu_launches": int(launches),
                "clocks": clocks,
                "roofline": {"kernel": dom, "bound": "tensor", "achieved": round(ach, 3), "peak": tf,
                             "unit": "TFLOP/s", "frac": round(ach / tf, 5), "peak_source": src, "traffic": None}}
        # config 3's long sequence: T = 32768 with an initial state and a final-state gradient (dh0 out)
        del W
        TL = 32768
        WL = Work(1, TL, 16, 32, 128, 128, 1, dev, args.algo, with_state=True)
        ms_l, per_op_l, launches_l, clocks_l = _timed(WL.step, args.steps, args.warmup, dev)
        dom_l = "layer_bwd" if "layer_bwd" in per_op_l else "gdn_bwd"
        ach_l = 2 * fpt * TL * 32 / (per_op_l[dom_l] / 1e3) / 1e12
        line["long_sequence"] = {
            "config": "config3's long sequence: B=1, T=32768, Hk=16 Hv=32 Dk=Dv=128, h0 and dh_T ~ N(0, 0.02), "
                      "dh0 returned", "value": round(TL / (ms_l / 1e3), 1), "unit": "tokens/s",
            "ms_per_step": round(ms_l, 4), "per_op_ms": {k: round(v, 4) for k, v in per_op_l.items()},
            "gpu_launches": int(launches_l), "clocks": clocks_l,
            "roofline": {"kernel": dom_l, "bound": "tensor", "achieved": round(ach_l, 3), "peak": tf,
                         "unit": "TFLOP/s", "frac": round(ach_l / tf, 5), "peak_source": src}}
    elif args.workload == "conv_norm":
        line = conv_norm_line(args, dev, hbm, src)
    else:
        N, V, Hk, Hv, D = 32, 8, 16, 32, 128
        p = synthetic.make(N, V, Hk, Hv, D, D, seed=0, device=dev, with_dy=False)
        q, k, v = p.q.to(torch.bfloat16), p.k.to(torch.bfloat16), p.v.to(torch.bfloat16)
        g, beta = p.g, p.beta
        gen = torch.Generator(device=dev).manual_seed(1)
        state = torch.randn(N, Hv, D, D, generator=gen, device=dev) * 0.05

        def step(events):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            exact.verify(q, k, v, g, beta, state)
            e1.record()
            if events is not None:
                events.append(("verify", e0, e1))

        ms, per_op, launches, clocks = _timed(step, args.steps, args.warmup, dev)
        rstates = exact.verify(q, k, v, g, beta, state)[1]
        decode = decode_line(args, dev, hbm, N, V, Hk, Hv, D, rstates)
        nbytes = (N * Hv * D * D * 4 + N * V * Hv * D * D * 4 + N * V * Hk * D * 2 * 2 + N * V * Hv * D * 2 * 2
                  + N * V * Hv * 4 * 2)
        ach = nbytes / (per_op["verify"] / 1e3) / 1e9
        line = {"metric": "exact speculative verify tokens/s", "value": round(N * V / (ms / 1e3), 1),
                "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded)",
                "config": {"workload": "config4: 32 sequences x 8 drafted tokens, Hk=16 Hv=32 Dk=Dv=128, "
                                       "every token's state kept", "l2": "flushed before every step"},
                "per_op_ms": {k: round(v, 4) for k, v in per_op.items()}, "gpu_launches": int(launches),
                "clocks": clocks,
                "roofline": {"kernel": "gdn_verify", "bound": "hbm", "achieved": round(ach, 1), "peak": hbm,
                             "unit": "GB/s", "frac": round(ach / hbm, 5), "peak_source": src,
                             "traffic": TRAFFIC.get(("c4", "verify")),
                             "bytes_per_launch": nbytes},
                "decode_integration": decode}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    elif a.workload in ("c3", "c4", "conv_norm"):
        run_single(a)
    else:
        run_ours(a)
