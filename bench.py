"""Benchmark of the MoE decode hot path (Qwen3-30B-A3B shape, Q4 experts).

A step is one decode step's MoE work: the MoE FFN of all 48 layers for B
tokens (router -> dispatch -> gate/up -> SwiGLU -> down -> combine per layer,
layers in sequence on one stream, as decode runs them). The metric is tokens
per second through that step (B / step time); the whole 15.4 GB Q4 store is
resident in HBM and every step streams each layer's active experts, so the
working set is far above the 126 MB L2 and no flush is needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B]
    python bench.py --impl reference ...   # the reference's CPU path, same metric

The headline batch is B=64 (the tensor-core path); the sweep adds B=1 (the
exact CUDA-core path, bit-identical to the reference), B=8 and B=32 in
`per_batch`. Output: one JSON line on rank 0 (see the keys below).
Multi-GPU (torchrun, N > 1) runs the layer expert-parallel: each GPU serves
its own B tokens and stores E/N experts; token rows and weighted outputs
cross GPUs as peer stores over NVLink by library kernels (--ep nccl: NCCL
all-to-all instead); weak scaling in tokens.
"""
from __future__ import annotations

import argparse
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

SHAPE = dict(d=2048, E=128, k=8, m=768, norm=1, L=48)
METRIC = "Qwen3-30B-A3B-shape Q4 MoE decode tok/s (48 MoE layers per step)"
TOL = 1e-3  # max row-relative error of expert outputs (north star)
DTYPE_TC = ("fp16 x fp16 -> fp32: Q4 weights dequantised to fp16 ((n-8)*s rounded), activations "
            "as fp16 hi + lo pairs, fp32 accumulate")
DTYPE_EXACT = "f32: Q4 weights, fp32 arithmetic in the reference's order"
DTYPE_GEMV = "f32: Q4 weights dequantised exactly, fp32 accumulate (another summation order)"


_T0 = time.time()


def log(msg: str) -> None:
    """Progress on stderr (the JSON line alone goes to stdout)."""
    print(f"[bench {time.time() - _T0:7.1f}s] {msg}", file=sys.stderr, flush=True)


def rec_bytes(d, m):
    return 3 * (m * d // 2 + m * d // 32)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region

class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.p, self.path = gpu, None, None

    def __enter__(self):
        try:
            import tempfile
            self.path = Path(tempfile.mkdtemp(prefix="joule_clocks_")) / f"clocks_gpu{self.gpu}.csv"
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()
            self.f.close()

    def summary(self):
        if not self.path or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# our arm

def dist_init():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(ws, v: float) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def build_store(moe, want_host_layers: int):
    """Quantise seeded N(0,0.02) weights on the device into every layer; keep a
    host copy (reference record layout) of the first `want_host_layers`."""
    import torch
    from joule_b200 import synth
    from joule_b200.native import get_dll
    cfg = moe.cfg
    E, d, m = cfg.E, cfg.d, cfg.intermediate
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(1)
    host = []
    L = get_dll()
    for l in range(cfg.L):
        gw = synth.router_bf16(E, d, gen, dev)
        ws = [torch.randn(E, m, d, generator=gen, device=dev) * 0.02,
              torch.randn(E, m, d, generator=gen, device=dev) * 0.02,
              torch.randn(E, d, m, generator=gen, device=dev) * 0.02]
        if l < want_host_layers:
            # reference-layout records on the device, then a host copy
            pk = [[None] * E for _ in range(3)]
            sc = [[None] * E for _ in range(3)]
            for p in range(3):
                n = m * d
                spk = torch.empty(E, n // 2, dtype=torch.uint8, device=dev)
                ssc = torch.empty(E, n // 64, dtype=torch.int16, device=dev)
                for e in range(E):
                    rc = L.jl_q4_quantize(ws[p][e].data_ptr(), n, ssc[e].data_ptr(), spk[e].data_ptr(),
                                          torch.cuda.current_stream().cuda_stream)
                    assert rc == 0
                hp, hs = spk.cpu().numpy(), ssc.cpu().numpy().view(np.uint16)
                for e in range(E):
                    pk[p][e], sc[p][e] = hp[e], hs[e]
            gwh = gw.cpu().numpy().view(np.uint16)
            moe.upload_layer(l, gwh, pk, sc)
            host.append((gwh, pk, sc))
        else:
            moe.quantize_layer(l, gw, *ws)
        del ws
    torch.cuda.synchronize()
    return host


def routing_unions(moe, xs, B):
    import torch
    U = []
    out = torch.empty(B, moe.cfg.d, device="cuda")
    for l in range(moe.cfg.L):
        moe.forward(l, xs[l, :B], out)
        U.append(moe.debug_routing(B)["U"])
    moe.check()
    return U


def capture_step(moe, xs, outs, B, mask, stream, layers):
    """One CUDA graph: `layers` consecutive layer forwards (phases in `mask`)."""
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            for l in layers:
                moe.forward_phases(l, xs[l, :B], outs[l, :B], mask, stream=stream)
    return g


def replay_ms(g, reps, warmup, stream, ws=1, preroll_s=0.0, reset=None):
    """Mean ms per replay of graph g: warm-up replays (at least `preroll_s`
    seconds of them, so that a clock sampler running over the warm-up and
    the timed region sees the GPU under this load), then `reps` replays back
    to back between two events (barrier + synchronize on both sides)."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
    stream.synchronize()
    t_start = time.perf_counter()
    while time.perf_counter() - t_start < preroll_s:
        if reset is not None:  # a graph with state that must not run past its buffers
            with torch.cuda.stream(stream):
                reset()
        with torch.cuda.stream(stream):
            for _ in range(4):
                g.replay()
        stream.synchronize()
    if reset is not None:
        with torch.cuda.stream(stream):
            reset()
        stream.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            g.replay()
    t1.record(stream)
    t1.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / reps


def time_batch(moe, xs, outs, B, steps, warmup, ws, phases=True, preroll_s=0.0):
    """The timed region: `steps` replays of the 48-layer step graph. Then each
    phase alone (48 back-to-back launches of one kernel, reading the routing
    the last full layer left) to attribute the time."""
    import torch
    L = moe.cfg.L
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for l in range(L):        # eager warm-up (kernel attributes are set outside capture)
            moe.forward(l, xs[l, :B], outs[l, :B], stream=stream)
    stream.synchronize()
    g = capture_step(moe, xs, outs, B, 7, stream, range(L))
    step_ms = replay_ms(g, steps, warmup, stream, ws, preroll_s)
    moe.check()
    phase = {}
    for name, mask in ((("router", 1), ("gateup", 2), ("down_combine", 4)) if phases else ()):
        gp = capture_step(moe, xs, outs, B, mask, stream, range(L))
        phase[name] = replay_ms(gp, max(3, steps // 2), 2, stream) / L
        del gp
    # leave the workspace consistent (full layers) for later users
    with torch.cuda.stream(stream):
        for l in range(L):
            moe.forward(l, xs[l, :B], outs[l, :B], stream=stream)
    stream.synchronize()
    moe.check()
    del g
    return step_ms * steps, phase


def e2e_dropin(host, B, steps, warmup, seed=11):
    """jl_layer_ffn_batch (the reference-facing C-ABI call, host buffers): one
    call per layer, each copying x in and out. Layers cycle over the host
    layers kept (all 48 when memory allows)."""
    import ctypes
    from joule_b200.moe import layer_ffn_batch
    from joule_b200.native import KernelCfg, KernelW
    d, E, k, m, L = SHAPE["d"], SHAPE["E"], SHAPE["k"], SHAPE["m"], SHAPE["L"]
    nl = len(host)
    cfg = KernelCfg(L=nl, d=d, E=E, topk=k, intermediate=m, norm_topk_prob=SHAPE["norm"])
    gate = np.ascontiguousarray(np.stack([h[0] for h in host]))
    keep = []
    W = KernelW()
    W.gate_w = gate.ctypes.data
    for p in range(3):
        pk = (ctypes.c_void_p * (nl * E))(*[host[l][1][p][e].ctypes.data for l in range(nl) for e in range(E)])
        sc = (ctypes.c_void_p * (nl * E))(*[host[l][2][p][e].ctypes.data for l in range(nl) for e in range(E)])
        keep += [pk, sc]
        W.expert_pk[p] = ctypes.cast(pk, ctypes.c_void_p)
        W.expert_sc[p] = ctypes.cast(sc, ctypes.c_void_p)
    rng = np.random.default_rng(seed)
    xs = rng.standard_normal((L, B, d)).astype(np.float32)
    out = np.empty((B, d), np.float32)
    for _ in range(max(warmup, 1)):
        for l in range(L):
            layer_ffn_batch(cfg, W, l % nl, xs[l], B, out)
    t = time.perf_counter()
    for _ in range(steps):
        for l in range(L):
            layer_ffn_batch(cfg, W, l % nl, xs[l], B, out)
    dt = (time.perf_counter() - t) / steps
    return dict(value=B / dt, unit="tok/s", h2d_bytes_per_step=L * B * d * 4,
                d2h_bytes_per_step=L * B * d * 4, ms_per_step=dt * 1e3,
                api="jl_layer_ffn_batch (host x/out, one call per layer)",
                host_layers=nl), keep


def cpu_moe_sample(B, budget_s=12.0):
    """The reference's layer_ffn_batch (oracle/_ref) on this host's cores: one
    seeded Qwen3-shape layer (bounded sample), extrapolated to the 48-layer
    step. Runs in a process of its own (run_isolated): the reference's thread
    pool cannot be started twice in one process."""
    from oracle import layer as olayer
    from oracle import ref
    if not ref.available():
        return None
    d, E, k, m, L = SHAPE["d"], SHAPE["E"], SHAPE["k"], SHAPE["m"], SHAPE["L"]
    lay = olayer.make_layer(d, E, k, m, SHAPE["norm"], seed_router=10, seed_experts=20)
    R = ref.RefLayer(lay)
    nthreads = ref_threads()
    R.L.spin_pool_init(nthreads)
    x = np.random.default_rng(5).standard_normal((B, d)).astype(np.float32)
    R.ffn(x)
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s and reps < 200:
        R.ffn(x)
        reps += 1
    t_layer = (time.perf_counter() - t0) / reps
    cores = 1 if B == 1 else nthreads + 1
    return dict(value=B / (t_layer * L), unit="tok/s", cores=cores, kind="reference",
                sample=f"1 Qwen3-shape MoE layer x {reps} calls of the reference's layer_ffn_batch at B={B} "
                       f"(16-token chunks), {t_layer * 1e3:.2f} ms/layer, x48 layers",
                threads_note="B=1 runs on one thread by the reference's design "
                             "(decode_kernel.c:1495-1497)" if B == 1 else
                             f"spin_pool_init({nthreads}) + main thread",
                cpu=cpu_model())


def cpu_decode_sample(B, budget_s=20.0, ctx=512, layers=2):
    """The reference's decode_layers_batch (oracle/_ref) on this host's cores:
    the Qwen3-30B-A3B shape with `layers` layers (seeded random weights, fp32
    lm_head of the full vocabulary), every sequence at position ctx over KV
    caches holding ctx rows (seeded random values, in place of a prefill of the
    reference's own, which would take minutes), B > 16 as 16-sequence calls
    (its BMAX). Timed with and without the lm_head (logits NULL), extrapolated
    to 48 layers + one lm_head per step. Runs in a process of its own."""
    import ctypes
    from oracle import decode as dec
    from oracle import ref
    if not ref.available():
        return None
    shape = dec.DecodeShape("qwen3_bench", layers, 2048, 32, 4, 128, 128, 8, 768, 151936, ctx + 8, 1, 0, 1,
                            1e-6, 1e6)
    model = dec.make_model(shape, 3)
    nthreads = ref_threads()
    r = dec.RefDecoder(model, threads=nthreads)
    caches = dec._Caches(shape, B)
    rng = np.random.default_rng(0)
    for arr in caches.k + caches.v:
        arr[:ctx] = rng.standard_normal((ctx, arr.shape[1]), dtype=np.float32)
    x = dec.embed(model, rng.integers(0, shape.V, B))
    logits = np.empty((16, shape.V), np.float32)
    P = ctypes.c_void_p

    def step(with_logits):
        for b0 in range(0, B, ref.BMAX):
            nb = min(ref.BMAX, B - b0)
            kv = (P * (2 * nb * layers))()
            for i in range(nb * layers):
                kv[2 * i] = caches.k[b0 * layers + i].ctypes.data
                kv[2 * i + 1] = caches.v[b0 * layers + i].ctypes.data
            pos = np.full(nb, ctx, np.int32)
            xs = np.ascontiguousarray(x[b0:b0 + nb])
            r.lib.decode_layers_batch(ctypes.byref(r.cfg), ctypes.byref(r.W), kv, pos.ctypes.data,
                                      xs.ctypes.data, nb, logits.ctypes.data if with_logits else None)

    def timed(with_logits):
        step(with_logits)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s / 2 and reps < 100:
            step(with_logits)
            reps += 1
        return (time.perf_counter() - t0) / reps, reps

    t_nolm, n1 = timed(False)
    t_lm, n2 = timed(True)
    t_layer = t_nolm / layers
    t_head = max(0.0, t_lm - t_nolm)
    t_step = SHAPE["L"] * t_layer + t_head
    return dict(value=B / t_step, unit="tok/s", cores=nthreads + 1, kind="reference",
                sample=f"the reference's decode_layers_batch, Qwen3 shape with {layers} layers, B={B} at "
                       f"position {ctx} (16-sequence calls): {t_layer * 1e3:.1f} ms per layer ({n1} steps), "
                       f"lm_head {t_head * 1e3:.1f} ms ({n2} steps); step = 48 layers + lm_head "
                       f"= {t_step * 1e3:.0f} ms",
                threads_note=f"spin_pool_init({nthreads}) + main thread", cpu=cpu_model())


def ref_threads() -> int:
    return max(1, min(16, (os.cpu_count() or 1) - 1))


def _isolated_child(fn_name, kwargs, q):
    sys.path.insert(0, str(ROOT))
    try:
        q.put(("ok", globals()[fn_name](**kwargs)))
    except Exception as e:  # reported, not raised: the baseline is optional
        q.put(("error", f"{type(e).__name__}: {e}"))


def run_isolated(fn_name, timeout_s=600, **kwargs):
    """Run one of this module's CPU-baseline functions in a spawned process."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_isolated_child, args=(fn_name, kwargs, q))
    p.start()
    try:
        status, res = q.get(timeout=timeout_s)
    except Exception:
        status, res = "error", "timed out"
    p.join(timeout=30)
    if p.is_alive():
        p.kill()
    return res if status == "ok" else {"unavailable": res}


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


def row_rel_err(out, ref) -> float:
    """max over rows of max|out - ref| / max|ref| (the north star's bar)."""
    import torch
    num = (out - ref).abs().amax(dim=1)
    den = ref.abs().amax(dim=1).clamp_min(1e-30)
    return float((num / den).max().item())


def run_ep(a, ws, rank, local):
    """N > 1: expert parallelism. Every rank serves its own B tokens (data
    parallel) and stores E/N experts of each layer; each layer exchanges token
    rows and weighted expert outputs with the experts' owners (library
    kernels over NVLink peer memory, or NCCL all-to-all with --ep nccl). Same
    seeded model as one GPU (each rank keeps its slice of the full weights).
    Before timing, layer 0's output on every rank is checked against a
    single-GPU forward of the same tokens on the exact path (the reference's
    arithmetic order): the run fails above 1e-3 max row-relative error."""
    import torch
    import torch.distributed as dist
    from joule_b200 import synth
    from joule_b200.ep import CudaEPBackend, ExpertParallelMoE
    from joule_b200.moe import PATH_EXACT, MoELayers, make_cfg
    d, E, k, m, L = SHAPE["d"], SHAPE["E"], SHAPE["k"], SHAPE["m"], SHAPE["L"]
    B = a.batch
    Bs = a.global_batch // ws if a.global_batch else 0  # strong scaling: fixed global batch
    Bcap = max(B, Bs)
    cfg = make_cfg(L, d, E, k, m, SHAPE["norm"])
    be = CudaEPBackend(cfg, Bcap, rank, ws)
    El = E // ws
    sl = slice(rank * El, (rank + 1) * El)
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(1)
    t = time.time()
    full0 = MoELayers(make_cfg(1, d, E, k, m, SHAPE["norm"]), B)  # layer 0, all experts: parity
    for l in range(L):
        gw = synth.router_bf16(E, d, gen, dev)
        w = [torch.randn(E, m, d, generator=gen, device=dev) * 0.02,
             torch.randn(E, m, d, generator=gen, device=dev) * 0.02,
             torch.randn(E, d, m, generator=gen, device=dev) * 0.02]
        be.quantize_layer(l, gw, *[t_[sl].contiguous() for t_ in w])
        if l == 0:
            full0.quantize_layer(0, gw, *w)
        del w
    torch.cuda.synchronize()
    setup_s = time.time() - t
    if a.ep == "p2p":
        from joule_b200.ep import P2PExpertParallelMoE
        ep = P2PExpertParallelMoE(be, Bcap)
    else:
        ep = ExpertParallelMoE(be, E)
    gx = torch.Generator(device=dev).manual_seed(100 + rank)
    xs = torch.randn(L, B, d, generator=gx, device=dev)

    # parity of the configuration timed below (layer 0, this rank's tokens)
    o_ep = ep.forward(0, xs[0]).clone()
    full0.set_path(PATH_EXACT)
    o_ref = full0.forward(0, xs[0])
    torch.cuda.synchronize()
    be.check()
    full0.check()
    err = torch.tensor([row_rel_err(o_ep, o_ref)], dtype=torch.float64, device=dev)
    dist.all_reduce(err, op=dist.ReduceOp.MAX)
    parity = dict(max_row_rel_err=float(err.item()), tokens_checked=ws * B, layer=0, tol=TOL,
                  against="single-GPU jl_moe_forward on the same tokens, exact path "
                          "(the reference's arithmetic order, bit-exact with its goldens)")
    full0.close()
    del o_ep, o_ref
    if parity["max_row_rel_err"] > TOL:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "error": "expert-parallel parity failed",
                              "parity": parity}), flush=True)
        dist.barrier()
        raise SystemExit(1)
    recv = []

    def step():
        for l in range(L):
            ep.forward(l, xs[l])
            if a.ep != "p2p":
                recv.append(sum(ep.last_counts))

    for _ in range(a.warmup):
        step()
    be.check()
    recv.clear()
    if a.ep == "p2p":
        ep.stats()  # reset the counters: only the timed steps count
    barrier(ws)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        tw0 = time.perf_counter()   # pre-roll: the sampler sees >= 1 s of this load
        while time.perf_counter() - tw0 < 1.0:
            step()
            torch.cuda.synchronize()
        barrier(ws)
        torch.cuda.synchronize()
        if a.ep == "p2p":
            ep.stats()
        recv.clear()
        t0.record()
        for _ in range(a.steps):
            step()
        t1.record()
        t1.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    ms = max_over_ranks(ws, t0.elapsed_time(t1))
    be.check()
    if a.ep == "p2p":
        nrows, ncalls = ep.stats()
        mean_rows = nrows / max(1, ncalls)
    else:
        mean_rows = float(np.mean(recv)) if recv else -1.0
    rows = torch.tensor([mean_rows], device=dev)
    rows_all = [torch.zeros_like(rows) for _ in range(ws)]
    dist.all_gather(rows_all, rows)

    # attribution (untimed): per-phase event times and the local union size of
    # every layer; bytes each rank streams from HBM and sends over NVLink
    phases = ["route", "order_send", "recv_wait", "dispatch", "gateup", "down", "return",
              "combine_wait"]
    Ul = []
    breakdown = None
    if a.ep == "p2p":
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(9)] for _ in range(L)]
        for l in range(L):
            ep.set_phase_events(evs[l])
            ep.forward(l, xs[l])
        ep.set_phase_events([])
        torch.cuda.synchronize()
        acc = np.zeros(8)
        for l in range(L):
            acc += [evs[l][i].elapsed_time(evs[l][i + 1]) * 1e3 for i in range(8)]
        mine = torch.tensor(acc / L, dtype=torch.float64, device=dev)
        allb = [torch.zeros_like(mine) for _ in range(ws)]
        dist.all_gather(allb, mine)
        breakdown = dict(unit="us per layer (mean over the 48 layers; CUDA events between "
                              "jl_ep_forward's kernels, untimed pass)",
                         phases=phases,
                         per_rank=[[round(float(v), 2) for v in b_.tolist()] for b_ in allb])
        Bpad = ws * B * k
        for l in range(L):
            ep.forward(l, xs[l])
            Ul.append(be.local.union_size(Bpad))
        be.check()
    e_bytes = (float(np.mean(Ul)) * rec_bytes(d, m) if Ul else None)
    us_layer = ms / a.steps * 1e3 / L
    roof = None
    if e_bytes is not None:
        hbm, peak_kind = peaks()
        layer_bytes = e_bytes + E * d * 2 + 2 * B * d * 4
        u_all = torch.tensor([layer_bytes], dtype=torch.float64, device=dev)
        dist.all_reduce(u_all, op=dist.ReduceOp.MAX)
        gbs = float(u_all.item()) / (us_layer * 1e-6) / 1e9
        nv = 2 * B * k * d * 4 * (ws - 1) / ws  # rows out and weighted rows back, remote share
        roof = dict(bound="hbm", kernel="whole expert-parallel layer on the busiest rank "
                                        "(its local experts' Q4 records + router rows + x/out)",
                    achieved=gbs, peak=hbm, unit="GB/s", frac=gbs / hbm, peak_kind=peak_kind,
                    traffic=None, algorithmic_bytes_per_layer=float(u_all.item()),
                    mean_local_union=float(np.mean(Ul)),
                    nvlink_bytes_per_layer_per_rank=nv,
                    nvlink_gbs=nv / (us_layer * 1e-6) / 1e9, nvlink_peak_gbs=770.0)
    # strong scaling: the global batch a.global_batch (256
    # sequences) split over the ranks, same layers
    strong = None
    if Bs >= 1:
        xs_s = torch.randn(L, Bs, d, generator=gx, device=dev)
        for _ in range(2):
            for l in range(L):
                ep.forward(l, xs_s[l])
        barrier(ws)
        torch.cuda.synchronize()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(a.steps):
            for l in range(L):
                ep.forward(l, xs_s[l])
        s1.record()
        s1.synchronize()
        barrier(ws)
        ms_s = max_over_ranks(ws, s0.elapsed_time(s1))
        be.check()
        strong = dict(global_batch=Bs * ws, batch_per_gpu=Bs, tok_s=Bs * ws * a.steps / (ms_s / 1e3),
                      ms_per_step=ms_s / a.steps, us_per_layer=ms_s / a.steps * 1e3 / L,
                      note="one GPU's point: moe_layer per_batch at B = global_batch in the N = 1 line")
        del xs_s
    # end to end: host x in, host out back, per layer
    xh = torch.randn(L, B, d, generator=torch.Generator().manual_seed(7 + rank)).pin_memory()
    oh = torch.empty(B, d).pin_memory()
    n_e2e = max(2, a.steps // 4)
    barrier(ws)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n_e2e):
        for l in range(L):
            o = ep.forward(l, xh[l].to(dev, non_blocking=True))
            oh.copy_(o, non_blocking=True)
    e1.record()
    e1.synchronize()
    barrier(ws)
    e2e_ms = max_over_ranks(ws, e0.elapsed_time(e1))
    val = ws * B * a.steps / (ms / 1e3)
    per_layer_launches = (2 if B > 32 else 1) + 6 + (3 if ws * B * k > 8 else 2)
    if rank == 0:
        line = dict(metric=METRIC, value=val, unit="tok/s", n_gpus=ws, steps=a.steps, warmup=a.warmup,
                    ms_per_step=ms / a.steps, higher_is_better=True, scaling="weak", vs_baseline=None,
                    dtype=DTYPE_TC,
                    data="synthetic: seeded N(0,0.02) weights quantised to the reference Q4 format, "
                         "x ~ N(0,1)",
                    config=dict(workload=f"Qwen3-30B-A3B-shape MoE FFN x48 layers, decode batch "
                                         f"{B} per GPU ({ws * B} total), expert parallel",
                                batch_per_gpu=B, global_batch=ws * B, layers=L, d=d, E=E, topk=k,
                                intermediate=m, norm_topk_prob=1, parallelism=f"ep{ws}",
                                experts_per_gpu=El,
                                exchange=("library kernels over NVLink peer memory (CUDA IPC): "
                                          "peer stores of token rows and weighted outputs, epoch "
                                          "flags, no host sync" if a.ep == "p2p" else
                                          "NCCL all_to_all_single of token rows and weighted outputs "
                                          "(torch.distributed), 3 per layer + counts"),
                                path="per rank: router (all E) then tensor-core or exact expert "
                                     "kernels on received rows (JL_PATH_AUTO)",
                                l2="not flushed: each step streams >= 1 GB of distinct expert weights",
                                store_setup_s=round(setup_s, 1)),
                    us_per_layer=us_layer,
                    parity=parity,
                    rows_received_per_layer=[round(float(r.item()), 1) for r in rows_all],
                    strong_scaling=strong,
                    ep_breakdown=breakdown,
                    clocks=clk.summary(),
                    gpu_launches=L * a.steps * per_layer_launches,
                    e2e=dict(value=ws * B * n_e2e / (e2e_ms / 1e3), unit="tok/s",
                             h2d_bytes_per_step=L * B * d * 4, d2h_bytes_per_step=L * B * d * 4,
                             api="ExpertParallelMoE.forward per layer, host x in / host out back"),
                    roofline=roof)
        print(json.dumps(line), flush=True)
    if a.ep == "p2p":
        dist.barrier()
        ep.close()
    be.close()
    dist.destroy_process_group()


def microbench(moe, a, hbm, peak_kind):
    """grouped expert microbenchmark. Tokens per step T in
    {1, 8, 64, 512, 4096}, Qwen3 MoE shape; routing logits log p + Gumbel
    with Zipf(1.2) popularity over a seeded permutation, fed through the
    router unchanged by router rows [I | 0] (logit_e = x_e). Each step runs
    the 48 layers (distinct expert weights; the routers are replaced)."""
    import torch
    from joule_b200 import synth
    d, E, k, m, L = SHAPE["d"], SHAPE["E"], SHAPE["k"], SHAPE["m"], SHAPE["L"]
    dev = torch.device("cuda", torch.cuda.current_device())
    Ts = [int(t) for t in a.micro.split(",")]
    Tmax = max(Ts)
    eye = synth.identity_router(E, d, dev)
    for l in range(L):
        moe.upload_router(l, eye)
    xs = torch.empty(L, Tmax, d, device=dev)
    g = torch.Generator(device=dev).manual_seed(300)
    for l in range(L):
        xs[l] = torch.randn(Tmax, d, generator=g, device=dev)
        xs[l, :, :E] = torch.from_numpy(synth.zipf_logits(Tmax, E, 1.2, seed=l)).to(dev)
    outs = torch.empty_like(xs)
    tensor_peak = tensor_peak_tflops()
    res = {}
    for T in Ts:
        log(f"microbench T={T}")
        U = routing_unions(moe, xs, T)
        total_ms, _ = time_batch(moe, xs, outs, T, max(3, a.steps // 2), 3, 1, phases=False)
        t_step = total_ms / max(3, a.steps // 2) / 1e3
        byts = sum(U) * rec_bytes(d, m) + L * (E * d * 2 + 2 * T * d * 4)
        flops = L * 2.0 * T * k * 3 * d * m
        t_hbm = byts / (hbm * 1e9)
        t_tc = flops / (tensor_peak * 1e12)
        res[str(T)] = dict(path=path_of(T), us_per_layer=t_step * 1e6 / L, tok_s=T / t_step,
                           mean_U=float(np.mean(U)), bytes_per_layer=byts / L, flops_per_layer=flops / L,
                           hbm_frac=t_hbm / t_step, tensor_frac=t_tc / t_step,
                           bound="hbm" if t_hbm >= t_tc else "tensor",
                           roofline_frac=max(t_hbm, t_tc) / t_step)
    return dict(config="BASELINE config 5: grouped expert microbenchmark, Zipf(1.2) routing "
                       "via router rows [I|0], 48 layers per step",
                peaks=dict(hbm_gbs=hbm, bf16_tflops=tensor_peak, kind=peak_kind),
                per_T=res)


def full_decode(a, hbm):
    """the whole decode step of the Qwen3-30B-A3B shape on
    one GPU (attention, norms, the 48 Q4 MoE layers, the lm_head and the
    argmax), seeded random-init weights built on the device. Context: every
    sequence's 512-token prompt of uniform-random ids runs through the same
    decode step first (all sequences batched, one step per position). Then
    greedy decode at each B: a step embeds the previous step's token, runs the
    decoder and takes the argmax, captured once as a CUDA graph (positions
    advance inside the graph). e2e: the token ids cross host <-> device every
    step (pinned host memory) with a synchronisation per step."""
    import torch
    from joule_b200.decoder import Decoder, qwen3_cfg
    Bs = sorted(set(int(b) for b in a.decode_sweep.split(",")))
    Bmax, ctx = max(Bs), a.ctx
    steps, warm = a.steps, a.warmup
    cfg = qwen3_cfg(maxT=ctx + warm + steps + 64)
    t0 = time.time()
    log("decoder build")
    dec = Decoder.random(cfg, Bmax, Bmax)
    build_s = time.time() - t0
    log(f"decoder built ({build_s:.1f}s); prefill {ctx} positions x {Bmax} sequences")
    dev = torch.device("cuda", torch.cuda.current_device())
    V, d, L = cfg.V, cfg.d, cfg.L
    prompt = torch.randint(0, V, (Bmax, ctx), generator=torch.Generator().manual_seed(0),
                           dtype=torch.int32).to(dev)
    slots = torch.arange(Bmax, dtype=torch.int32, device=dev)
    x = torch.empty(Bmax, d, device=dev)
    tok0 = torch.empty(Bmax, dtype=torch.int32, device=dev)
    t0 = time.time()
    for p in range(ctx):
        pos = torch.full((Bmax,), p, dtype=torch.int32, device=dev)
        dec.embed(prompt[:, p].contiguous(), x)
        dec.step(slots, pos, x, tok=tok0 if p == ctx - 1 else None)
    torch.cuda.synchronize()
    dec.check()
    prefill_s = time.time() - t0
    res = {}
    clocks = None
    stream = torch.cuda.Stream()
    for B in [b for b in Bs if b != a.batch] + ([a.batch] if a.batch in Bs else []):
        log(f"full decode B={B}")
        pos = torch.full((B,), ctx, dtype=torch.int32, device=dev)
        tok = tok0[:B].clone()
        xb = torch.empty(B, d, device=dev)
        sl = slots[:B].contiguous()
        with torch.cuda.stream(stream):  # eager once (sets kernel attributes outside capture)
            dec.embed(tok, xb, stream=stream)
            dec.step(sl, pos, xb, tok=tok, stream=stream)
        stream.synchronize()
        pos.fill_(ctx)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                dec.embed(tok, xb, stream=stream)
                dec.step(sl, pos, xb, tok=tok, stream=stream)
                pos.add_(1)
        if B == a.batch:  # the headline: clocks sampled over >= 1 s of replays, then the timed region
            with Clocks(torch.cuda.current_device()) as clk:
                ms = replay_ms(g, steps, warm, stream, preroll_s=1.0, reset=lambda: pos.fill_(ctx))
            clocks = clk.summary()
        else:
            ms = replay_ms(g, steps, warm, stream)
        dec.check(stream)
        # end to end: token ids host -> device -> host each step
        tok_h = torch.empty(B, dtype=torch.int32).pin_memory()
        tok_h.copy_(tok.cpu())
        pos.fill_(ctx)
        n_e2e = max(3, steps // 2)
        stream.synchronize()
        e0 = time.perf_counter()
        for _ in range(n_e2e):
            with torch.cuda.stream(stream):
                tok.copy_(tok_h, non_blocking=True)
                g.replay()
                tok_h.copy_(tok, non_blocking=True)
            stream.synchronize()
        e2e_s = (time.perf_counter() - e0) / n_e2e
        dec.check(stream)
        del g
        res[str(B)] = dict(tok_s=B / (ms / 1e3), ms_per_step=ms,
                           e2e=dict(value=B / e2e_s, unit="tok/s", h2d_bytes_per_step=B * 4,
                                    d2h_bytes_per_step=B * 4, ms_per_step=e2e_s * 1e3,
                                    api="Decoder.embed + Decoder.step (jl_dec_embed, jl_dec_step) as one "
                                        "CUDA graph, token ids host->device and back every step"))
    dec.close()
    torch.cuda.synchronize()
    return dict(clocks=clocks, config="BASELINE config 3: Qwen3-30B-A3B architecture, random-init (bf16 dense N(0,0.02), "
                       "fp32 lm_head, Q4 experts), 48 layers, GQA 32/4 x 128, per-head QK-norm, RoPE theta "
                       "1e6, eps 1e-6, vocab 151936; context 512 uniform-random ids (seed 0) then greedy decode",
                context=ctx, build_s=round(build_s, 1), prefill_s=round(prefill_s, 1),
                path="norms, attention, projections and lm_head in the reference's fp32 order on CUDA cores "
                     "(register-tiled matvecs from B = 16); MoE layers JL_PATH_AUTO (GEMV path for B <= 4, "
                     "tensor cores above)",
                per_batch=res)


def tensor_peak_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def run_ours(a):
    import torch
    from joule_b200.moe import MoELayers, make_cfg
    SHAPE["L"] = a.layers
    ws, rank, local = dist_init()
    if ws > 1:
        return run_ep(a, ws, rank, local)
    d, E, k, m, L = SHAPE["d"], SHAPE["E"], SHAPE["k"], SHAPE["m"], SHAPE["L"]
    sweep = sorted(set(int(b) for b in a.sweep.split(",")) | {a.batch})
    Bmax = max(sweep + ([max(int(t) for t in a.micro.split(","))] if a.micro else []))
    moe = MoELayers(make_cfg(L, d, E, k, m, SHAPE["norm"]), Bmax)
    host_layers = L if a.e2e else 1
    t = time.time()
    host = build_store(moe, host_layers)
    setup_s = time.time() - t
    log(f"store built ({setup_s:.1f}s)")
    gen = torch.Generator(device="cuda").manual_seed(100 + rank)
    Bs = max(sweep)
    xs = torch.randn(L, Bs, d, generator=gen, device="cuda")
    outs = torch.empty_like(xs)
    hbm, peak_kind = peaks()
    per_b = {}
    head = None
    clocks = None
    # the headline batch runs last, with the clocks sampled over >= 1 s of
    # warm-up replays and then its timed region
    for B in [b for b in sweep if b != a.batch] + [a.batch]:
        log(f"moe layer B={B}")
        U = routing_unions(moe, xs, B)
        if B == a.batch:
            with Clocks(local) as clk:
                total_ms, phase = time_batch(moe, xs, outs, B, a.steps, a.warmup, ws, preroll_s=1.0)
            clocks = clk.summary()
        else:
            total_ms, phase = time_batch(moe, xs, outs, B, a.steps, a.warmup, ws)
        ms_step = total_ms / a.steps
        layer_bytes = [u * rec_bytes(d, m) + E * d * 2 + 2 * B * d * 4 for u in U]
        gu_bytes = [u * 2 * (m * d // 2 + m * d // 32) + B * d * 4 + B * k * m * 4 for u in U]
        rec = dict(
            path=path_of(B),
            tok_s=B * a.steps / (total_ms / 1e3), ms_per_step=ms_step,
            us_per_layer=ms_step * 1e3 / L, mean_U=float(np.mean(U)),
            layer_gbs=sum(layer_bytes) / (ms_step / 1e3) / 1e9,
            phase_us={k: v * 1e3 for k, v in phase.items()},
            gateup_gbs=float(np.mean(gu_bytes)) / (phase["gateup"] / 1e3) / 1e9,
            gateup_bytes_per_launch=float(np.mean(gu_bytes)))
        rec["layer_frac_of_hbm"] = rec["layer_gbs"] / hbm
        rec["gateup_frac_of_hbm"] = rec["gateup_gbs"] / hbm
        per_b[str(B)] = rec
        if B == a.batch:
            head = rec
    line = dict(metric=METRIC, value=head["tok_s"], unit="tok/s", n_gpus=ws, steps=a.steps,
                warmup=a.warmup, ms_per_step=head["ms_per_step"], higher_is_better=True,
                scaling="weak", vs_baseline=None,
                dtype=dtype_of(a.batch),
                data="synthetic: seeded N(0,0.02) weights quantised to the reference Q4 format, "
                     "x ~ N(0,1)",
                config=dict(workload=f"Qwen3-30B-A3B-shape MoE FFN x48 layers, decode batch B={a.batch}",
                            batch=a.batch, layers=L, d=d, E=E, topk=k, intermediate=m,
                            norm_topk_prob=1,
                            path=("gemv (warp-per-row GEMVs over every SM, fp32 in another order; "
                                  "<= 1e-3 row-relative)"
                                  if path_of(a.batch) == "gemv" else
                                  "tensor-core (tcgen05 grouped GEMM, fp16 weights x fp16 hi+lo "
                                  "activations, fp32 accumulate; <= 1e-3 row-relative)"),
                            l2="not flushed: each step streams >= 1 GB of distinct expert weights "
                               "(store 15.4 GB) vs 126 MB L2",
                            parallelism="single GPU",
                            store_setup_s=round(setup_s, 1)),
                per_batch=per_b)
    kern = gateup_kernel(a.batch)
    line["roofline"] = dict(bound="hbm",
                            kernel=f"{kern} (gate + up rows of the union experts, SwiGLU fused; "
                                   f"phase time includes {'nothing else' if kern == 'k_gateup_gemv' else 'the token permute'})",
                            achieved=head["gateup_gbs"], peak=hbm, unit="GB/s",
                            frac=head["gateup_gbs"] / hbm, peak_kind=peak_kind,
                            traffic=traffic_from_profiles(kern, a.batch),
                            algorithmic_bytes_per_launch=head["gateup_bytes_per_launch"],
                            layer_gbs=head["layer_gbs"], layer_frac=head["layer_gbs"] / hbm)
    line["clocks"] = clocks
    line["gpu_launches"] = launches_per_step(a.batch) * a.steps
    if a.e2e:
        log("e2e drop-in")
        e2e, keep = e2e_dropin(host, a.batch, max(2, a.steps // 4), 1)
        line["e2e"] = e2e
    if a.cpu:
        cb = {}
        for B in sorted({1, a.batch}):
            log(f"cpu moe sample B={B}")
            c = run_isolated("cpu_moe_sample", B=B)
            if c is not None and "value" in c:
                cb[str(B)] = c
                if str(B) in per_b:
                    per_b[str(B)]["cpu_tok_s"] = c["value"]
                    per_b[str(B)]["gpu_over_cpu"] = per_b[str(B)]["tok_s"] / c["value"]
        line["cpu_baseline"] = cb.get(str(a.batch))
        line["cpu_baseline_per_batch"] = cb
    if a.micro:
        log("microbench")
        line["microbench"] = microbench(moe, a, hbm, peak_kind)
    if a.decode_sweep:
        moe.close()
        del xs, outs
        torch.cuda.empty_cache()
        fd = full_decode(a, hbm)
        if str(a.batch) in fd["per_batch"]:
            line = decode_headline(a, line, fd)
    print(json.dumps(line), flush=True)


METRIC_DECODE = ("Qwen3-30B-A3B-shape Q4 decode tok/s (full model: 48 layers of attention + Q4 MoE, "
                 "lm_head, greedy argmax)")


def decode_headline(a, line, fd):
    """The full-model decode step is the headline (BASELINE metric: decode
    tok/s); the MoE-layer measurements move under `moe_layer`, and the roofline
    stays on the dominant kernel (the MoE gate/up kernel)."""
    moe_keys = ("metric", "value", "ms_per_step", "dtype", "config", "per_batch", "e2e", "cpu_baseline",
                "cpu_baseline_per_batch", "clocks", "gpu_launches")
    moe = {k: line.pop(k) for k in moe_keys if k in line}
    head = fd["per_batch"][str(a.batch)]
    L = SHAPE["L"]
    moe_launches = launches_per_step(a.batch) // L
    out = dict(metric=METRIC_DECODE, value=head["tok_s"], unit="tok/s", n_gpus=1, steps=a.steps,
               warmup=a.warmup, ms_per_step=head["ms_per_step"], higher_is_better=True, scaling="weak",
               vs_baseline=None,
               dtype=("f32 (attention, norms, projections, lm_head in the reference's fp32 order); MoE: "
                      + dtype_of(a.batch)),
               data="synthetic: seeded random-init weights (bf16 dense N(0,0.02), fp32 lm_head, Q4 experts "
                    "quantised from N(0,0.02)), 512-token contexts of uniform-random ids",
               config=dict(workload=f"Qwen3-30B-A3B decode step, batch B={a.batch} at context {a.ctx}",
                           model="Qwen3-30B-A3B architecture, random init (BASELINE config 3)",
                           batch=a.batch, context=a.ctx, layers=L,
                           l2="not flushed: each step streams the 3.7 GB of dense weights and the active "
                              "experts of 48 layers vs 126 MB L2",
                           parallelism="single GPU"),
               e2e=head["e2e"], clocks=fd.get("clocks"),
               gpu_launches=(L * (dense_launches(a.batch) + moe_launches) + 5) * a.steps,
               full_decode=fd)
    for k in ("roofline", "microbench"):
        if k in line:
            out[k] = line.pop(k)
    moe.update(line)
    out["moe_layer"] = moe
    if a.cpu:
        cb = {}
        for B in sorted({1, a.batch}):
            log(f"cpu decode sample B={B}")
            c = run_isolated("cpu_decode_sample", timeout_s=900, B=B, ctx=a.ctx)
            if c is not None and "value" in c:
                cb[str(B)] = c
                if str(B) in fd["per_batch"]:
                    fd["per_batch"][str(B)]["cpu_tok_s"] = c["value"]
        out["cpu_baseline"] = cb.get(str(a.batch))
        out["cpu_baseline_per_batch"] = cb
    return out


def path_of(B):
    """The path jl_moe_forward takes (JL_PATH_AUTO) at batch B for this shape."""
    return "gemv" if B <= 4 else "tensor-core"


def dtype_of(B):
    return DTYPE_GEMV if path_of(B) == "gemv" else DTYPE_TC


def gateup_kernel(B):
    return "k_gateup_gemv" if path_of(B) == "gemv" else "k_expert_tc<false>"


def dense_launches(B):
    # per layer outside the MoE layer: two norms, QKV, o_proj and the attention:
    # k_attn_qk + k_attn_pv below B = 16, k_qk_prep + k_attn_qk_t + k_attn_pv_t from 16
    # (the Qwen3 shape: head dim 128, groups of 8 heads)
    return 4 + (3 if B >= 16 else 2)


def launches_per_step(B):
    # per layer: the cluster router (routing, and the dispatch for B <= 32),
    # k_dispatch_fast for B > 32, then
    #   gemv: gate/up, down, combine; tensor-core: permute, gate/up, down, combine
    return SHAPE["L"] * (1 + (1 if B > 32 else 0) + (3 if path_of(B) == "gemv" else 4))


def traffic_from_profiles(kernel, B):
    """DRAM bytes (read + write) per launch of `kernel` at batch B from the
    committed ncu summary (profiles/traffic.txt lines `kernel B=<B> = <bytes>`)."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith(f"{kernel} B={B} "):
            return float(line.split("=")[2].split()[0])
    return None


# ---------------------------------------------------------------------------
# reference arm: the reference's own CPU path on this host's cores

def run_reference(a):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import layer as olayer
    from oracle import ref
    if not ref.available():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libjoule_ref.so not built (needs the reference sources)"}))
        return
    d, E, k, m, L = SHAPE["d"], SHAPE["E"], SHAPE["k"], SHAPE["m"], SHAPE["L"]
    if ws == 1 and a.decode_sweep:
        # the headline metric at N = 1: the whole decode step (our arm's full_decode)
        budget = min(240.0, max(20.0, 4.0 * (a.steps + a.warmup)))
        c = cpu_decode_sample(a.batch, budget_s=budget, ctx=a.ctx)
        line = dict(metric=METRIC_DECODE, value=c["value"], unit="tok/s", n_gpus=1, steps=a.steps,
                    warmup=a.warmup, ms_per_step=a.batch / c["value"] * 1e3, higher_is_better=True,
                    scaling="weak", vs_baseline=None, dtype=DTYPE_EXACT, impl="reference",
                    data="synthetic: seeded random-init weights in the reference's layout (bf16 dense, fp32 "
                         "lm_head, Q4 experts), KV caches of 512 seeded random rows",
                    config=dict(workload=f"Qwen3-30B-A3B decode step, batch B={a.batch} at context {a.ctx}",
                                model="Qwen3-30B-A3B architecture, random init (BASELINE config 3)",
                                batch=a.batch, context=a.ctx, layers=L),
                    cpu_baseline=c,
                    e2e=dict(value=c["value"], unit="tok/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
        print(json.dumps(line), flush=True)
        return
    nl = a.ref_layers
    t = time.time()
    lays = [olayer.make_layer(d, E, k, m, SHAPE["norm"], seed_router=10 + i, seed_experts=20 + i)
            for i in range(nl)]
    setup = time.time() - t
    ncores = os.cpu_count() or 1
    nthreads = max(1, min(16, ncores - 1))
    R = [ref.RefLayer(lay) for lay in lays]
    R[0].L.spin_pool_init(nthreads)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((a.batch, d)).astype(np.float32)
    for _ in range(a.warmup):
        for r in R:
            r.ffn(x)
    times = []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        for r in R:
            r.ffn(x)
        times.append(time.perf_counter() - t0)
    R[0].L.spin_pool_shutdown()
    t_layer = float(np.mean(times)) / nl
    step = t_layer * L
    val = a.batch / step
    cores = 1 if a.batch == 1 else nthreads + 1
    line = dict(metric=METRIC, value=val, unit="tok/s", n_gpus=ws, steps=a.steps, warmup=a.warmup,
                ms_per_step=step * 1e3, higher_is_better=True, scaling="weak", vs_baseline=None,
                dtype=DTYPE_EXACT, impl="reference",
                data="synthetic: seeded N(0,0.02) weights in the reference Q4 format, x ~ N(0,1)",
                config=dict(workload=f"Qwen3-30B-A3B-shape MoE FFN x48 layers, decode batch B={a.batch}",
                            batch=a.batch, layers=L, d=d, E=E, topk=k, intermediate=m,
                            norm_topk_prob=1, store_setup_s=round(setup, 1)),
                cpu_baseline=dict(value=val, unit="tok/s", cores=cores, kind="reference",
                                  sample=f"each step = {nl} distinct Qwen3-shape layers through the "
                                         f"reference's layer_ffn_batch (B>16 as 16-token calls), "
                                         f"time x{L}/{nl}",
                                  cpu=cpu_model(), threads=nthreads),
                e2e=dict(value=val, unit="tok/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--sweep", default="1,8,32,64,256")
    ap.add_argument("--global-batch", type=int, default=256,
                    help="N > 1: also time this global batch split over the ranks (strong scaling; 0: off)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-layers", type=int, default=2)
    ap.add_argument("--layers", type=int, default=48, help="MoE layers per step (48 = the model)")
    ap.add_argument("--no-e2e", dest="e2e", action="store_false")
    ap.add_argument("--no-cpu", dest="cpu", action="store_false")
    ap.add_argument("--micro", default="1,8,64,512,4096",
                    help="config 5 token counts ('' to skip the microbenchmark)")
    ap.add_argument("--decode-sweep", default="1,8,32,64",
                    help="full-model decode batch sizes (config 3; '' to skip)")
    ap.add_argument("--ctx", type=int, default=512, help="context before the timed decode steps")
    ap.add_argument("--ep", default="p2p", choices=["p2p", "nccl"],
                    help="N > 1 exchange: library peer-memory kernels or NCCL all-to-all")
    a = ap.parse_args()
    if a.warmup < 3:
        a.warmup = 3
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
