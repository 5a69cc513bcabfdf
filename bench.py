#!/usr/bin/env python
"""bench.py — MoE-layer decode throughput of libmoe_cuda on B200.

Workload: one Qwen3-30B-A3B-shaped MoE layer,
hidden 2048, 128 experts, moe_intermediate 768, top-8, Q8 experts, decode of
T tokens (default 16; T=1 and T=4 are reported beside it). A "step" is one
moe_ffn call (router -> top-k -> routed experts -> k-ordered combine +
residual) on one batch of T tokens. Steps rotate through NL resident layers
(default 16, 9.7 GB of Q8 experts) and a pool of input batches, so every step
streams its experts from HBM (a layer's routed experts plus the other layers'
exceed the 126 MB L2 between two visits of the same layer).

Synthetic data: random-init weights of the real shapes (seeded, see
moe.cc_b200/synth.py), hidden states ~ N(0,1).

N>1 (torchrun): expert parallelism, rank r holds experts [r*128/N, (r+1)*128/N)
and routes its own T tokens (weak scaling: T tokens per GPU). The default
exchange is fused into the kernels (moe_ffn_ep): the routing kernel stores
each rank's truncated activations and top-k into every peer's buffers, the
down projection's epilogue stores each slot row straight into the owning
rank's buffer, and a flag-synchronised combine finishes each rank's tokens.
MOE_EP_EXCHANGE=nccl selects the NCCL decomposition instead (all-gather of
the tokens, moe_ffn_partial, reduce-scatter of the slot rows, combine).

--impl reference: the reference's own C (kernels.c + test_model_trace.c MoE
block, compiled from source into oracle/_ref; else this repo's C port) on the
host cores, same metric and config. That arm loads nothing of the product:
its inputs come from the oracle's copy of the seeded input stream.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "moe.cc_b200"))

E, D, F, TOPK = 128, 2048, 768, 8
METRIC = "MoE-layer decode tok/s (Q8, Qwen3-30B-A3B layer shape)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--dtype", default="q8", choices=["q8", "q4"])
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--extra-t", default="1,4", help="other T values reported beside the headline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemv-c1", action="store_true", help="skip the configs[0] batched GEMV line")
    ap.add_argument("--no-full-model", action="store_true",
                    help="skip the configs[3] and configs[4] 48-layer decodes through the C host driver")
    ap.add_argument("--prefill-t", default="512,2048",
                    help="configs[2] Q4 prefill sizes reported beside the headline ('' to skip)")
    ap.add_argument("--q4-batch", type=int, default=32,
                    help="configs[4]: Q4 batched decode of this many tokens per step over all GPUs "
                         "(strong scaling; 0 to skip)")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), \
        int(os.environ.get("LOCAL_RANK", 0))


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed
    region: NVML every 10 ms (nvidia-smi every 200 ms if NVML is missing)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_index):
        self.idx, self.stop = gpu_index, threading.Event()
        self.sm, self.reasons, self.max_mhz = [], set(), None
        self.th = threading.Thread(target=self.run, daemon=True)
        self.nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[gpu_index]) if vis and vis.split(",")[gpu_index].isdigit() else gpu_index
            self.h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
            self.nvml = pynvml
        except Exception:
            self.nvml = None

    def sample(self):
        if self.nvml is not None:
            n = self.nvml
            self.sm.append(float(n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM)))
            r = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            self.reasons |= {k for k, b in self.BITS.items() if r & b}
            return
        out = subprocess.run(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                              "--format=csv,noheader,nounits"], capture_output=True,
                             text=True, timeout=5).stdout.strip()
        if out:
            row = [c.strip() for c in out.split(",")]
            if row[1].replace(".", "").isdigit():
                self.sm.append(float(row[1]))
            if self.max_mhz is None and row[2].replace(".", "").isdigit():
                self.max_mhz = float(row[2])
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            self.reasons |= {nm for nm, v in zip(names, row[5:9]) if v.strip() == "Active"}

    def run(self):
        while not self.stop.is_set():
            try:
                self.sample()
            except Exception:
                pass
            self.stop.wait(0.01 if self.nvml is not None else 0.2)

    def __enter__(self):
        self.th.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        self.th.join(timeout=10)

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        sm = sorted(self.sm)
        return {"sm_mhz": sm[len(sm) // 2], "sm_min_mhz": sm[0], "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(sm),
                "source": "nvml" if self.nvml is not None else "nvidia-smi"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_table():
    """Per-launch DRAM bytes of each kernel from a committed ncu summary, if any."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f)
    except Exception:
        return {}


def alg_bytes(kernel, T, U, dt):
    """Algorithmic HBM bytes of one launch (weights + scales read once, token
    activations in/out). U = distinct experts routed in that step."""
    gu_rb = D if dt == 2 else D // 2
    d_rb = F if dt == 2 else F // 2
    kernel = (kernel.replace("mma_", "").replace("down_ep", "down").replace("ep_combine", "combine")
              .replace("route_dispatch", "route").replace("fused_ep", "fused"))
    if kernel == "fused":      # gate/up and down in one persistent kernel
        return alg_bytes("gateup", T, U, dt) + alg_bytes("down", T, U, dt)
    if kernel == "gateup":
        return U * (2 * F * gu_rb + 2 * F * 4)
    if kernel == "down":
        return U * (D * d_rb + D * 4)
    if kernel in ("router_logits", "route"):
        return E * D * 4 + T * D * 4 + T * E * 4
    if kernel == "combine":
        return T * TOPK * D * 4 + 2 * T * D * 4    # slot outputs in, residual in, result out
    return None


def layer_bytes_step(T, U, dt):
    return sum(alg_bytes(k, T, U, dt) for k in ("route", "gateup", "down", "combine"))


def build_layers(torch, mc, sy, nl, dt, base=0):
    for l in range(nl):
        Ld = sy.make_layer_dev(torch, 1, l, E, D, F, dt, bias=False)
        mc.upload_layer(base + l, Ld, device_arrays=True)
        del Ld
    torch.cuda.synchronize()
    mc.check_status()


def make_inputs(torch, mc, T, pool, seed):
    xs, xa = [], []
    for i in range(pool):
        a = torch.empty(T, D, device="cuda")
        b = torch.empty(T, D, device="cuda")
        mc.synth_normal_dev(seed * 7919 + 2 * i, a, 1.0)
        mc.synth_normal_dev(seed * 7919 + 2 * i + 1, b, 1.0)
        xs.append(a); xa.append(b)
    return xs, xa


class Runner:
    """One decode step on this rank.

    N=1: moe_ffn on the T resident tokens.
    N>1 (expert parallel, T tokens per rank): all-gather the ranks' tokens,
    moe_ffn_partial on all T*N tokens (every rank routes all of them; each
    computes only its own experts' slots), reduce-scatter the slot outputs so
    each rank receives its own tokens' slots (exactly one rank contributes each
    slot, so the sum is exact), then the k-ordered combine + residual.
    With MOE_EP_EXCHANGE=fused (the default when every rank has its own GPU)
    the step is one moe_ffn_ep call and no collective: the routing kernel
    sends this rank's tokens and top-k to every rank, the down GEMM's
    epilogue stores each slot row into the owning rank's buffer over NVLink,
    and kernels synchronise on flags in peer memory.
    """

    def __init__(self, torch, mc, dist, world, rank, T, nl, pool, base=0, ep_ready=False):
        self.torch, self.mc, self.dist, self.world, self.rank = torch, mc, dist, world, rank
        self.T, self.nl, self.base = T, nl, base
        self.xs, self.xa = make_inputs(torch, mc, T, pool, seed=T * 131 + rank)
        self.out = [x.clone() for x in self.xa]
        self.stream = torch.cuda.current_stream()
        if world > 1:
            TN = T * world
            self.x_all = torch.empty(TN, D, device="cuda")
            self.y_all = torch.empty(TN * TOPK, D, device="cuda")
            self.p_all = torch.empty(TN, TOPK, device="cuda")
            self.y_loc = torch.empty(T * TOPK, D, device="cuda")
            own_gpu = torch.cuda.device_count() >= world
            self.fused = os.environ.get("MOE_EP_EXCHANGE", "fused" if own_gpu else "nccl") == "fused"
            if self.fused and not ep_ready:
                handles = [None] * world
                dist.all_gather_object(handles, mc.ep_setup(T, D, TOPK))
                mc.ep_connect(handles)
                dist.barrier()

    def step(self, i, topk_idx=None, x_in=None, out=None):
        j = i % len(self.xs)
        layer = self.base + i % self.nl
        x = self.xs[j] if x_in is None else x_in
        o = self.out[j] if out is None else out
        if self.world == 1:
            self.mc.moe_ffn_dev(layer, x, o, topk_idx, None, stream=self.stream)
        elif self.fused and topk_idx is None:
            self.mc.moe_ffn_ep(layer, x, o, stream=self.stream)
        else:
            self.dist.all_gather_into_tensor(self.x_all, x)
            self.mc.moe_ffn_partial(layer, self.x_all, self.y_all, topk_idx, self.p_all, stream=self.stream)
            self.dist.reduce_scatter_tensor(self.y_loc, self.y_all)
            p = self.p_all[self.rank * self.T:(self.rank + 1) * self.T]
            self.mc.moe_ffn_combine(self.y_loc, p, o, TOPK, stream=self.stream)

    def _bracket(self):
        self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def _max_over_ranks(self, ms):
        if self.world > 1:
            t = self.torch.tensor([ms], device="cuda")
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def timed(self, steps, warmup):
        torch = self.torch
        for i in range(warmup):
            self.step(i)
        self._bracket()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        for i in range(steps):
            self.step(warmup + i)
        b.record(self.stream)
        self._bracket()
        ms = self._max_over_ranks(a.elapsed_time(b))
        self.mc.check_status()
        return ms

    def timed_host(self, steps, warmup):
        """Same steps with the tokens coming from pinned host memory and the
        result going back to it, copies inside the timed region (N>1 e2e)."""
        torch = self.torch
        hx = [torch.empty(self.T, D).pin_memory() for _ in range(4)]
        for i, h in enumerate(hx):
            h.copy_(self.xs[i].cpu())
        ho = torch.empty(self.T, D).pin_memory()
        xd, od = torch.empty(self.T, D, device="cuda"), torch.empty(self.T, D, device="cuda")

        def one(i):
            xd.copy_(hx[i % 4], non_blocking=True)
            od.copy_(self.xa[i % len(self.xa)])
            self.step(i, x_in=xd, out=od)
            ho.copy_(od, non_blocking=True)
        for i in range(warmup):
            one(i)
        self._bracket()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        for i in range(steps):
            one(warmup + i)
        b.record(self.stream)
        self._bracket()
        return self._max_over_ranks(a.elapsed_time(b))

    def distinct_experts(self, steps, warmup):
        """Distinct experts this rank computes per step (routing is a pure
        function of layer and input)."""
        torch = self.torch
        TN = self.T * self.world
        idx = torch.empty(steps, TN, TOPK, dtype=torch.int32, device="cuda")
        for i in range(steps):
            self.step(warmup + i, idx[i])
        torch.cuda.synchronize()
        h = idx.cpu().numpy()
        lo, hi = E * self.rank // self.world, E * (self.rank + 1) // self.world
        return [len({e for e in h[i].ravel().tolist() if lo <= e < hi}) for i in range(steps)]


def e2e_host(torch, mc, T, steps, warmup, nl):
    """Same metric through the C-ABI with pinned HOST buffers: every step copies
    x_norm2 and x_inout in, the result and top-k out (inside the timed region)."""
    import numpy as np
    xs = [torch.from_numpy(mc.synth_normal_host(5000 + i, T * D, 1.0).reshape(T, D)).pin_memory()
          for i in range(8)]
    xo = [torch.from_numpy(mc.synth_normal_host(6000 + i, T * D, 1.0).reshape(T, D)).pin_memory()
          for i in range(8)]
    idx = torch.empty(T, TOPK, dtype=torch.int32).pin_memory()
    p = torch.empty(T, TOPK, dtype=torch.float32).pin_memory()
    lib = mc.lib()
    # the buffers' addresses resolved once, as a C caller holds them; every
    # step still passes host buffers through the C-ABI and copies in and out
    xs_p = [x.data_ptr() for x in xs]
    xo_p = [x.data_ptr() for x in xo]
    idx_p, p_p, ffn = idx.data_ptr(), p.data_ptr(), lib.moe_ffn

    def call(i):
        rc = ffn(i % nl, xs_p[i % 8], xo_p[i % 8], T, idx_p, p_p, mc.HOST_PTRS, None)
        if rc:
            mc.check(rc)
    for i in range(warmup):
        call(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(torch.cuda.default_stream())
    for i in range(steps):
        call(warmup + i)
    b.record(torch.cuda.default_stream())
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    return {"value": T * steps / (ms / 1e3), "unit": "tok/s",
            "h2d_bytes_per_step": 2 * T * D * 4, "d2h_bytes_per_step": T * D * 4 + T * TOPK * 8,
            "ms_per_step": ms / steps}


def host_layer_from_device(torch, mc, sy, dt):
    """Layer 0 rebuilt on the GPU and copied to host numpy (CPU-baseline input)."""
    Ld = sy.make_layer_dev(torch, 1, 0, E, D, F, dt, bias=False)
    torch.cuda.synchronize()
    L = {k: (v.cpu().numpy() if hasattr(v, "cpu") else v) for k, v in Ld.items()}
    L["topk"] = TOPK
    L.setdefault("router_b", None)
    return L


def host_layer(gen, dt):
    """Layer 0 built on the host (no GPU), same seeds as synth.make_layer_dev.
    gen(seed, n, std) draws the seeded normal stream: the product's
    moe_synth_normal_host for the product arm's CPU baseline, the oracle's
    restatement of it for the reference arm (which loads nothing of the
    product). The streams are equal bit for bit (tests/test_oracle_cpu.py)."""
    import numpy as np
    from oracle.oracle import Port
    port = Port()
    L = {"dtype": dt, "topk": TOPK, "router_b": None,
         "router_w": gen(_stream_seed(1, 0, 0), E * D, 0.02).reshape(E, D)}
    shapes = {"g": (F, D), "u": (F, D), "d": (D, F)}
    for j, nm in enumerate("gud"):
        rows, cols = shapes[nm]
        qs, ss = [], []
        for e in range(E):
            w = gen(_stream_seed(1, 0, 2 + 3 * e + j), rows * cols, 0.02)
            q, s = port.quantize(w.reshape(rows, cols), dt)
            qs.append(q); ss.append(s)
        L[nm + "q"] = np.ascontiguousarray(np.stack(qs))
        L[nm + "s"] = np.ascontiguousarray(np.stack(ss))
    return L


def _stream_seed(seed, layer, tid):
    """synth.stream_seed, repeated here so the reference arm need not import
    the product's Python package."""
    return (seed * 1_000_003 + layer * 1009 + tid) & ((1 << 64) - 1)


def cpu_engine():
    from oracle.oracle import Port, Ref
    if Ref.available():
        return "reference", Ref()
    return "port", Port()


def cpu_step(kind, eng, L, xn, xa):
    if kind == "reference":
        # the reference's layer_forward_f32 with zero attention: MoE input = rmsnorm(x)
        eng.moe_layer(xa, L)
    else:
        eng.moe_block(xn, xa, L)


def cpu_baseline(gen, L, T, budget_s=12.0):
    """The reference's own CPU path (oracle/_ref, single-threaded as shipped) on a
    bounded sample of the same workload: whole T-token steps until ~budget_s."""
    kind, eng = cpu_engine()
    n, t0 = 0, time.perf_counter()
    while True:
        xn = gen(7000 + n, T * D, 1.0).reshape(T, D)
        xa = gen(7500 + n, T * D, 1.0).reshape(T, D)
        cpu_step(kind, eng, L, xn, xa)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    cores = 1 if kind == "reference" else (os.cpu_count() or 1)
    return {"value": n * T / dt, "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"{n} steps of T={T} tokens (one Q8 layer each), {dt:.1f} s"}


def _ref_worker(kind, eng, L, xs, quota, deadline, ready, go, out):
    """One host process of the reference arm: its own copy of the reference's
    library state (globals, profiler tables), whole T-token steps until its
    quota or the shared deadline."""
    cpu_step(kind, eng, L, *xs[0])              # warm-up inside the process
    ready.wait()
    go.wait()
    n, t0 = 0, time.perf_counter()
    while n < quota and time.perf_counter() < deadline.value:
        cpu_step(kind, eng, L, *xs[n % len(xs)])
        n += 1
    out.put((n, time.perf_counter() - t0))


def run_reference(args, budget_s=150.0):
    """The reference's own CPU path (oracle/_ref: its kernels.c and
    layer_forward_f32, single-threaded as shipped) on every host core the
    process may use: one forked process per core, each running whole T-token
    steps of the same layer, the K requested steps shared among them. The
    timed region runs until the K steps are done or budget_s has passed (then
    `steps` reports the steps actually run). value = tokens of all processes
    / wall time of the timed region."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import multiprocessing as mp
    from oracle.oracle import Port
    gen = Port().synth_normal        # the oracle's copy of the input stream
    dt = 2 if args.dtype == "q8" else 3
    L = host_layer(gen, dt)
    kind, eng = cpu_engine()
    T = args.tokens
    xs = [(gen(7000 + i, T * D, 1.0).reshape(T, D),
           gen(7500 + i, T * D, 1.0).reshape(T, D)) for i in range(4)]
    for i in range(args.warmup):
        cpu_step(kind, eng, L, *xs[i % 4])
    try:
        avail = len(os.sched_getaffinity(0))
    except AttributeError:
        avail = os.cpu_count() or 1
    # the C restatement parallelises inside (OpenMP); the reference runs one
    # thread per process
    procs = max(1, min(avail, args.steps)) if kind == "reference" else 1
    ctx = mp.get_context("fork")
    ready, go = ctx.Barrier(procs + 1), ctx.Barrier(procs + 1)
    deadline = ctx.Value("d", 0.0)
    out = ctx.Queue()
    quotas = [args.steps // procs + (1 if p < args.steps % procs else 0) for p in range(procs)]
    ws = [ctx.Process(target=_ref_worker, args=(kind, eng, L, xs[p % 4:] + xs[:p % 4], quotas[p], deadline,
                                                 ready, go, out)) for p in range(procs)]
    for w in ws:
        w.start()
    ready.wait()
    deadline.value = time.perf_counter() + budget_s
    t0 = time.perf_counter()
    go.wait()
    res = [out.get() for _ in ws]
    sec = time.perf_counter() - t0
    for w in ws:
        w.join()
    done = sum(n for n, _ in res)
    v = T * done / sec
    cores = procs if kind == "reference" else (os.cpu_count() or 1)
    sample = (f"{done} timed steps of T={T} (one Q8 layer each) over {procs} host processes"
              if dt == 2 else f"{done} timed steps of T={T} (one Q4 layer each) over {procs} host processes")
    if done < args.steps:
        sample += f"; capped at {budget_s:.0f} s of the {args.steps} requested"
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": done, "warmup": args.warmup, "ms_per_step": sec * 1e3 / max(done, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int32-acc q8" if dt == 2 else "int32-acc q4", "data": "synthetic",
            "config": {"workload": f"configs[1]: Qwen3-30B-A3B MoE layer decode, T={T} per GPU",
                       "tokens": T, "experts": E, "hidden": D, "moe_intermediate": F, "top_k": TOPK},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def gemv_c1(torch, mc, sy, peak, reps=50, warmup=5):
    """BASELINE configs[0] (the reference's own CPU kernel path, one Q8/Q4
    768x2048 matvec), in the batched form that can fill the GPU: all 128
    experts' gate matrices against one x[2048] in one moe_matmul_batched_dev
    call (201 MB Q8, 101 MB Q4). Two such sets alternate, so each call reads
    its matrices from HBM. A call is two launches: the activation
    quantisation and the GEMV. Algorithmic bytes: weights + scales + x + C."""
    N, K, nm = 768, 2048, 128
    st = torch.cuda.current_stream()
    out = {}
    for dt, name in ((mc.Q8, "q8"), (mc.Q4, "q4")):
        rb = K if dt == mc.Q8 else K // 2
        tmp = torch.empty(N, K, dtype=torch.float32, device="cuda")
        sets = []
        for s in range(2):
            q = torch.empty(nm, N, rb, dtype=torch.int8 if dt == mc.Q8 else torch.uint8, device="cuda")
            sc = torch.empty(nm, N, dtype=torch.float32, device="cuda")
            for e in range(nm):
                mc.synth_normal_dev(sy.stream_seed(1, s, 2 + 3 * e), tmp, 0.02, stream=st)
                mc.quantize_rowwise_dev(tmp, q[e], sc[e], dt, stream=st)
            qp = torch.tensor([q[e].data_ptr() for e in range(nm)], dtype=torch.int64, device="cuda")
            sp = torch.tensor([sc[e].data_ptr() for e in range(nm)], dtype=torch.int64, device="cuda")
            sets.append((q, sc, qp, sp))
        x = torch.empty(1, K, dtype=torch.float32, device="cuda")
        mc.synth_normal_dev(sy.stream_seed(2, 0, 0), x, 1.0, stream=st)
        C = torch.empty(nm, N, dtype=torch.float32, device="cuda")

        def call(i):
            _, _, qp, sp = sets[i % 2]
            mc.check(mc.lib().moe_matmul_batched_dev(x.data_ptr(), qp.data_ptr(), sp.data_ptr(), C.data_ptr(),
                                                     nm, N, K, dt, st.cuda_stream))
        for i in range(warmup):
            call(i)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for i in range(reps):
            call(i)
        b.record(st)
        torch.cuda.synchronize()
        mc.check_status()
        us = a.elapsed_time(b) * 1e3 / reps
        byts = nm * (N * rb + 4 * N) + 4 * K + 4 * nm * N
        out[name] = {"matrices": nm, "N": N, "K": K, "us_per_call": us, "alg_bytes": byts,
                     "gb_s": byts / (us * 1e-6) / 1e9, "frac_hbm": byts / (us * 1e-6) / 1e9 / peak,
                     "launches_per_call": 2}
        del sets, tmp, C
    return out


def full_model_c4(layers=48, prompt=64, steps=16, timeout_s=300):
    """BASELINE configs[3] through the C host driver (moe.cc_b200/moe_generate):
    the 48-layer Qwen3-30B-A3B-shaped model with random-init weights and Q8
    experts, a 64-token prompt, then greedy decode. Attention, norms and the
    head run on the host (fp32), the MoE block of every layer on the GPU; the
    figure of interest is the MoE wall time per layer call (host pointers,
    copies included). Decodes `steps` of configs[3]'s 256 tokens to bound the
    run time. Runs as its own process."""
    import subprocess
    tool = os.path.join(ROOT, "moe.cc_b200", "moe_generate")
    r = subprocess.run([tool, "--layers", str(layers), "--prompt", str(prompt), "--steps", str(steps),
                        "--dtype", "q8"], capture_output=True, text=True, timeout=timeout_s)
    if r.returncode != 0:
        return {"error": (r.stderr or r.stdout)[-300:]}
    out = json.loads(r.stdout.strip().splitlines()[-1])
    out["workload"] = (f"configs[3]: 48-layer decoder, Q8 experts, batch 1, {prompt}-token prompt, "
                       f"{steps} of the 256 greedy tokens")
    return out


def c5_context(world, layers=48, batch=32):
    """The largest context of 8192, 4096, 2048, 1024 whose host memory (every
    rank's KV cache, fp32 attention weights, embedding and head) fits in half
    of the memory available now."""
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        avail = 64 << 30
    per_rank_weights = 4 * (layers * (4096 * 2048 * 2 + 512 * 2048 * 2) + 2 * 151936 * 2048)
    for ctx in (8192, 4096, 2048, 1024):
        kv = 2 * 4 * layers * batch * ctx * 512
        if kv + world * per_rank_weights <= avail // 2:
            return ctx
    return 512


def full_model_c5(world, rank, local, dist, steps=3, timeout_s=600):
    """BASELINE configs[4] through the C host driver: the 48-layer model with
    Q4 experts, 32 sequences decoding in lockstep at a long context (every
    KV cache prefilled with N(0,1)), one token per sequence per step, the
    experts sharded over the N GPUs (moe_ffn_ep in every MoE block, 32/N
    sequences per rank). Runs as one moe_generate process per GPU; the bench
    processes only wait for them (no GPU work meanwhile). The context is the
    largest of 8192/4096/2048/1024 that fits host memory (c5_context)."""
    import subprocess
    import tempfile
    ctx = c5_context(world)
    tool = os.path.join(ROOT, "moe.cc_b200", "moe_generate")
    cmd = [tool, "--layers", "48", "--dtype", "q4", "--batch", "32", "--kv-fill", str(ctx), "--prompt", "1",
           "--steps", str(steps + 1)]
    env = dict(os.environ)
    tmp = None
    if world > 1:
        box = [tempfile.mkdtemp(prefix="moe_ep_") if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tmp = box[0]
        cmd += ["--ep-dir", tmp]
        env.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(local), NCCL_NVLS_ENABLE="0")
        # torchrun pins OMP_NUM_THREADS=1 for its ranks; the host attention of
        # each moe_generate rank gets an equal share of the cores instead
        try:
            ncpu = len(os.sched_getaffinity(0))
        except AttributeError:
            ncpu = os.cpu_count() or 1
        env["OMP_NUM_THREADS"] = str(max(1, ncpu // world))
    else:
        cmd += ["--device", str(local)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s, env=env)
    except subprocess.TimeoutExpired:
        return {"error": f"moe_generate did not finish within {timeout_s} s"}
    if r.returncode != 0:
        return {"error": (r.stderr or r.stdout)[-300:]}
    if rank != 0:
        return None
    out = json.loads(r.stdout.strip().splitlines()[-1])
    out["workload"] = (f"configs[4]: 48-layer decoder, Q4 experts, 32 sequences in lockstep at context {ctx} "
                       f"(KV prefilled N(0,1)), experts sharded over {world} GPU(s) by expert parallelism")
    out["context"] = ctx
    if world > 1:
        out["note"] = ("moe_ms_per_layer_call includes waiting for the slowest rank's host attention: "
                       "the ranks' MoE calls run in lockstep")
    out["context_rule"] = "largest of 8192/4096/2048/1024 whose host KV cache and weights fit half of free memory"
    return out


def prefill_bench(torch, mc, sy, steps, warmup, ts):
    """the same layer with Q4 experts, prefill of T tokens,
    router logits skewed by a seeded per-expert bias ~ N(0,1) (ragged expert
    loads). Four resident Q4 layers (each 304 MB > L2), steps rotate over them.
    Reported beside the decode headline; the expert GEMMs' tensor throughput is
    the grouped-GEMM evidence (int8 MMAs, counted as 2 ops per MAC)."""
    ids = [1000 + i for i in range(4)]
    for k, lid in enumerate(ids):
        Ld = sy.make_layer_dev(torch, 3, k, E, D, F, 3, bias=True)
        mc.upload_layer(lid, Ld, device_arrays=True)
        del Ld
    torch.cuda.synchronize()
    out = {}
    for T in ts:
        xs = [sy.make_tokens_dev(torch, 4000 + T + i, T, D) for i in range(4)]
        xo = [x.clone() for x in xs]
        st = torch.cuda.current_stream()

        def run(n, w0):
            for i in range(n):
                j = (w0 + i) % 4
                mc.moe_ffn_dev(ids[j], xs[j], xo[j], stream=st)
        run(warmup, 0)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        run(steps, warmup)
        b.record(st)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        mc.profile(True)
        run(steps, 0)
        prof = mc.profile_read()
        mc.profile(False)
        mc.check_status()
        kern = {n: v[0] / max(v[1], 1) * 1e3 for n, v in prof.items()}
        mac = T * TOPK * 3 * F * D                      # gate + up + down MACs
        gemm_us = kern.get("mma_gateup", 0) + kern.get("mma_down", 0)
        out[f"T{T}"] = {"tok_s": T / (ms / 1e3), "us_per_step": ms * 1e3,
                        "kernels_us": {n: round(v, 1) for n, v in kern.items()},
                        "gemm_tops_int8": 2 * mac / (gemm_us * 1e-6) / 1e12 if gemm_us else None,
                        "gemm_us": gemm_us}
    for lid in ids:
        mc.free_layer(lid)
    return out


def run_ours(args):
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    import moe_cuda as mc
    import synth as sy
    mc.init(local, world, rank)
    dt = 2 if args.dtype == "q8" else 3
    nl = args.layers
    build_layers(torch, mc, sy, nl, dt)
    T = args.tokens
    steps, warmup = args.steps, max(args.warmup, 3)
    pool = 64

    run = Runner(torch, mc, dist, world, rank, T, nl, pool)
    with ClockSampler(local) as clk:
        ms = run.timed(steps, warmup)
    clocks = clk.summary()
    TN = T * world                       # tokens per step over all ranks
    value = TN * steps / (ms / 1e3)

    # routed experts per step and per-kernel device times (separate profiled pass)
    Us = run.distinct_experts(min(steps, 64), warmup)
    U = sum(Us) / len(Us)
    mc.profile(True)
    run.timed(steps, 0)
    prof = mc.profile_read()
    mc.profile(False)
    peak, peak_kind = peaks()
    kern = {}
    for name, (tot, cnt) in prof.items():
        avg_ms = tot / max(cnt, 1)
        b = alg_bytes(name, TN if name == "route" else T, U, dt)
        kern[name] = {"avg_us": avg_ms * 1e3, "launches": cnt,
                      "share": tot / max(sum(v[0] for v in prof.values()), 1e-9),
                      "alg_bytes": b, "gbs": (b / (avg_ms * 1e-3) / 1e9) if b else None}
    dom = max((k for k in kern if kern[k]["alg_bytes"]), key=lambda k: kern[k]["share"])
    tr = traffic_table().get(f"{dom}_T{T}_{args.dtype}")
    roof = {"kernel": dom, "bound": "hbm", "achieved": kern[dom]["gbs"], "peak": peak,
            "unit": "GB/s", "frac": kern[dom]["gbs"] / peak, "peak_source": peak_kind,
            "traffic": tr, "alg_bytes_per_launch": kern[dom]["alg_bytes"]}
    layer_gbs = layer_bytes_step(T, U, dt) / (ms / steps * 1e-3) / 1e9   # this rank's bytes
    launches_per_step = sum(v["launches"] for v in kern.values()) / steps

    extra = {}
    if world == 1:
        for t in [int(v) for v in args.extra_t.split(",") if v]:
            if t == T:
                continue
            r2 = Runner(torch, mc, dist, world, rank, t, nl, pool)
            ms2 = r2.timed(steps, warmup)
            u2 = r2.distinct_experts(min(steps, 64), warmup)
            extra[f"T{t}"] = {"tok_s": t * steps / (ms2 / 1e3), "us_per_step": ms2 * 1e3 / steps,
                              "distinct_experts": sum(u2) / len(u2),
                              "layer_gbs": layer_bytes_step(t, sum(u2) / len(u2), dt)
                              / (ms2 / steps * 1e-3) / 1e9}
    if world == 1:
        e2e = e2e_host(torch, mc, T, steps, warmup, nl)
    else:
        ms_h = run.timed_host(steps, warmup)
        e2e = {"value": TN * steps / (ms_h / 1e3), "unit": "tok/s",
               "h2d_bytes_per_step": T * D * 4, "d2h_bytes_per_step": T * D * 4,
               "ms_per_step": ms_h / steps, "note": "per rank: tokens in from pinned host, result out"}
    # Q4 experts, batched decode of q4_batch sequences per step, the
    # experts sharded over the ranks (strong scaling: q4_batch / N tokens per rank)
    q4b = None
    if args.q4_batch and args.q4_batch % world == 0 and (world == 1 or args.q4_batch // world <= T):
        nlq = 8
        try:
            build_layers(torch, mc, sy, nlq, 3, base=1000)
            r4 = Runner(torch, mc, dist, world, rank, args.q4_batch // world, nlq, 16, base=1000, ep_ready=True)
            ms4 = r4.timed(steps, warmup)
        except Exception as exc:       # the headline line must still be printed
            ms4, q4b = None, {"error": str(exc)[:300]}
    if q4b is None and args.q4_batch and args.q4_batch % world == 0 and (world == 1 or args.q4_batch // world <= T):
        q4b = {"workload": f"configs[4]: Q4 experts, batched decode of {args.q4_batch} tokens per step, "
                           f"experts sharded over {world} GPU(s)",
               "tokens_per_step": args.q4_batch, "tokens_per_gpu": args.q4_batch // world,
               "tok_s": args.q4_batch * steps / (ms4 / 1e3), "us_per_step": ms4 * 1e3 / steps,
               "scaling": "strong", "resident_layers": nlq,
               "exchange": None if world == 1 else ("fused peer stores" if r4.fused else "nccl")}
    prefill = None
    if world == 1 and args.prefill_t:
        prefill = prefill_bench(torch, mc, sy, 30, 3, [int(v) for v in args.prefill_t.split(",") if v])
    c1 = None
    if world == 1 and not args.no_gemv_c1:
        try:
            c1 = gemv_c1(torch, mc, sy, peak)
        except Exception as exc:       # the headline line must still be printed
            c1 = {"error": str(exc)[:300]}
    c4 = None
    if world == 1 and not args.no_full_model:
        try:
            c4 = full_model_c4()
        except Exception as exc:       # the headline line must still be printed
            c4 = {"error": str(exc)[:300]}
    c5 = None
    if not args.no_full_model:
        try:
            c5 = full_model_c5(world, rank, local, dist)
        except Exception as exc:       # the headline line must still be printed
            c5 = {"error": str(exc)[:300]}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(mc.synth_normal_host, host_layer_from_device(torch, mc, sy, dt), T)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
                "steps": steps, "warmup": warmup, "ms_per_step": ms / steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int32-acc q8" if dt == 2 else "int32-acc q4", "data": "synthetic",
                "config": {"workload": f"configs[1]: Qwen3-30B-A3B MoE layer decode, T={T} per GPU",
                           "tokens": T, "tokens_per_step": TN, "experts": E, "hidden": D, "moe_intermediate": F,
                           "top_k": TOPK, "resident_layers": nl, "input_pool": pool,
                           "parallelism": f"ep{world}",
                           "ep_exchange": (None if world == 1 else
                                           ("fused peer stores" if run.fused else "nccl reduce_scatter")),
                           "l2": "inputs larger than L2: steps rotate over resident layers"},
                "roofline": roof,
                "layer": {"alg_gbs": layer_gbs, "frac_hbm": layer_gbs / peak,
                          "distinct_experts": U, "us_per_step": ms * 1e3 / steps},
                "kernels": kern, "gpu_launches": int(round(launches_per_step * steps)),
                "gpu_launches_per_step": launches_per_step,
                "clocks": clocks, "e2e": e2e, "cpu_baseline": cpu, "extra": extra,
                "prefill_q4": prefill, "q4_batch32": q4b, "gemv_c1": c1, "full_model_q8": c4,
                "full_model_q4_batch32": c5}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
