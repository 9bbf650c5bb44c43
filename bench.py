"""Benchmark of the fused block-sparse attention hot path (selection + forward +
backward) on B200, following the driver contract.

Workload (BASELINE config 3a, the north star): B=1, H=8, N=262144, D=64,
block 64, top-16 content blocks + the own block (kk=17), causal, bf16.
One step = mean-pooled block selection + fused forward + fused backward over
synthetic N(0,1) inputs resident in HBM.  With --gpus N the heads are sharded
over the ranks (H/N heads each, no collective: every head is independent), so
the total work is fixed ("strong" scaling); value = tokens of the whole job
per second, timed on the device as the max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --config {2,3b,4,5} [--n N]     the other BASELINE configurations
                                                   (one JSON line each, not the driver line)

The driver line also carries two sub-objects timed in the same run (max over
ranks, strong scaling):
  qsharded_262k  the same 262k step with the sequence split by query blocks
                 (NCCL all-gathers of K, V, the pooled summaries and the
                 selection rows; fp32 reduce-scatter of dK/dV);
  long_fwd       BASELINE config 3b at 16M tokens (block 128, forward only),
                 query-block sharded, with the peak allocation beside the size an
                 nblk x nblk score matrix would take.

--impl reference times the CPU restatement of the reference's gather path
(oracle/, the reference is Python and cannot be installed on the GPU box) on
a bounded sample of the same workload, with all host threads.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "fused-block-sparse-attention_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "fwd+bwd tokens/s at 262k tok (selection+forward+backward)"
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per step of each phase
# at N=262144, summed over the phase's kernels in one ncu launch-list capture of
# this bench (cold cache), and the source revision that capture was taken at.
# A recorded figure, not measured by this run: it is printed with its revision so
# that a stale figure is visible.
TRAFFIC_262K = {"attn_bwd": 14.70e9, "attn_fwd": 1.16e9, "select": 0.57e9}
TRAFFIC_REV = "23a77c5"
UNIT = "tokens/s"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def workload(a):
    H = 8
    cfg = dict(B=1, H=H, N=a.n, D=64, bs=64, topk=16, dtype="bf16", causal=True)
    cfg["nblk"] = cfg["N"] // cfg["bs"]
    cfg["kk"] = cfg["topk"] + 1
    return cfg


def config_dict(cfg, world):
    """The `config` object of the driver line (identical in both arms)."""
    return {"workload": "BASELINE config 3a: selection+fwd+bwd, B1 H8 N%d D64 block64 top16 (+own) "
                        "causal" % cfg["N"],
            "B": cfg["B"], "H": cfg["H"], "N": cfg["N"], "D": cfg["D"], "block": cfg["bs"],
            "kk": cfg["kk"], "parallelism": "heads sharded %d/rank" % (cfg["H"] // world),
            "l2": "256 MB buffer written between timed steps; inputs %.0f MB per rank"
                  % (4 * cfg["B"] * (cfg["H"] // world) * cfg["N"] * cfg["D"] * 2 / 1e6)}


def flops(cfg, heads):
    """Algorithmic FLOPs (FA2 5-GEMM convention): fwd 4*B*H*N*kk*bs*D, bwd 2.5x fwd,
    selection 2*D per causal block pair plus the two pooling passes (negligible)."""
    fwd = 4.0 * cfg["B"] * heads * cfg["N"] * cfg["kk"] * cfg["bs"] * cfg["D"]
    nb = cfg["nblk"]
    sel = 2.0 * cfg["D"] * cfg["B"] * heads * nb * (nb - 1) / 2
    return fwd, 2.5 * fwd, sel


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons every 20 ms while the timed loop
    runs.  The sampler starts half a second before the timed region (nvidia-smi
    needs that long to come up) and only the samples whose timestamps fall inside
    the region are summarised, so idle samples around it do not count."""

    def __init__(self, index, enabled=True):
        self.index = index
        self.enabled = enabled  # only the printing rank samples; every rank waits alike
        self.proc = None
        self.t0 = self.t1 = None
        self.path = os.path.join(tempfile.gettempdir(), "bsa_bench_clocks_%d_%d.csv" % (index, os.getpid()))

    def __enter__(self):
        q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            if not self.enabled:
                raise RuntimeError("sampling off on this rank")
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + q,
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.5)
        self.t0 = time.time()
        return self

    def __exit__(self, *exc):
        self.t1 = time.time()
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()
            self.f.close()

    def summary(self):
        import datetime
        if self.proc is None or not os.path.exists(self.path):
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(f[2]), float(f[3]), f[6:10]))
            except ValueError:
                continue
        inside = [r for r in rows if self.t0 - 0.02 <= r[0] <= self.t1 + 0.02]
        if not inside:
            return None
        reasons = set()
        for r in inside:
            for n, v in zip(names, r[3]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": inside[-1][2],
                "reasons": sorted(reasons), "samples": len(inside),
                "window_ms": round((self.t1 - self.t0) * 1e3, 1)}


# ---------------------------------------------------------------- our arm
def make_inputs(cfg, heads, h0, dev):
    """Seeded N(0,1) q, k, v, dO of the local heads (one generator per head, so the
    data of a head does not depend on the rank count)."""
    B, N, D = cfg["B"], cfg["N"], cfg["D"]
    out = []
    for name in range(4):
        t = torch.empty(B, heads, N, D, dtype=torch.bfloat16, device=dev)
        for j in range(heads):
            g = torch.Generator(device=dev).manual_seed(1000 * (h0 + j) + name)
            t[:, j].copy_(torch.randn(B, N, D, generator=g, device=dev))
        out.append(t)
    return out


def step(cfg, q, k, v, do, ph=None):
    """selection + forward + backward through the C ABI; ph: events per phase."""
    import _bsa
    import selection
    bs, causal = cfg["bs"], cfg["causal"]
    if ph:
        ph[0].record()
    sel, _, _ = selection.select_meanpool(q, k, bs=bs, topk=cfg["topk"], causal=causal)
    if ph:
        ph[1].record()
    o, lse = _bsa.attn_fwd(q, k, v, sel, None, bs=bs, causal=causal)
    if ph:
        ph[2].record()
    dq, dk, dv, _ = _bsa.attn_bwd(q, k, v, o, do, sel, lse, None, bs=bs, causal=causal)
    if ph:
        ph[3].record()
    return o, dq, dk, dv


def count_launches(cfg, q, k, v, do):
    """Kernels of this library launched by one step (torch profiler / CUPTI)."""
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step(cfg, q, k, v, do)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    ours = [n for n in names if "bsa::" in n or "cub::" in n or "bsa" in n.split("(")[0]]
    return len(ours), sorted(set(n.split("(")[0][:60] for n in ours))


def e2e_run(cfg, heads, q, k, v, do, steps, warmup):
    """Same step through the public drop-in API with host buffers: every step copies
    its q, k, v, dO in from pinned host memory, runs selection + bsattn forward and
    backward, and copies o, dq, dk, dv back out.  Copies run on their own streams
    and overlap the neighbouring steps' compute (inputs double-buffered on the
    device, outputs double-buffered on the host); the timed region spans the first
    step's input copy to the last step's output copy."""
    import selection
    import triton_kernel as tk
    hs = [t.cpu().pin_memory() for t in (q, k, v, do)]
    outs = [[torch.empty_like(h).pin_memory() for h in hs] for _ in range(2)]
    dev_in = [[torch.empty_like(t) for t in (q, k, v, do)] for _ in range(2)]
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    in_ready = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]

    def upload(buf):
        with torch.cuda.stream(up):
            up.wait_event(used[buf])
            for d, h in zip(dev_in[buf], hs):
                d.copy_(h, non_blocking=True)
            in_ready[buf].record(up)

    def compute(buf):
        comp.wait_event(in_ready[buf])
        qd, kd, vd, dod = (t.detach() for t in dev_in[buf])
        sel, _, _ = selection.select_meanpool(qd, kd, bs=cfg["bs"], topk=cfg["topk"])
        qd.requires_grad_(True)
        kd.requires_grad_(True)
        vd.requires_grad_(True)
        o = tk.bsattn(qd, kd, vd, sel, None, causal=cfg["causal"])
        o.backward(dod)
        res = [o.detach(), qd.grad, kd.grad, vd.grad]
        used[buf].record(comp)
        return res

    def download(buf, res):
        with torch.cuda.stream(down):
            down.wait_event(used[buf])
            for h, d in zip(outs[buf], res):
                h.copy_(d, non_blocking=True)
                d.record_stream(down)

    def run(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload((i + 1) % 2)
            res = compute(i % 2)
            download(i % 2, res)

    for e in used:
        e.record(comp)
    run(warmup)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(up)
    run(steps)
    e1.record(down)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    nbytes = sum(t.numel() * t.element_size() for t in hs)
    return ms, nbytes, sum(t.numel() * t.element_size() for t in outs[0])


def run_ours(a):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    cfg = workload(a)
    if cfg["H"] % world:
        raise SystemExit("H=%d heads cannot be split over %d ranks" % (cfg["H"], world))
    heads = cfg["H"] // world
    h0 = rank * heads
    q, k, v, do = make_inputs(cfg, heads, h0, dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)   # 256 MB > 126 MB L2

    for _ in range(a.warmup):
        step(cfg, q, k, v, do)
    torch.cuda.synchronize()
    if a.kernels_only:
        # profiling runs (ncu): the timed steps only, no profiler, copies or CPU legs
        for _ in range(a.steps):
            step(cfg, q, k, v, do)
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"kernels_only": True, "steps": a.steps, "warmup": a.warmup}))
        if dist:
            dist.destroy_process_group()
        return
    nlaunch, kernel_names = count_launches(cfg, q, k, v, do)

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(a.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local, enabled=rank == 0) as clk:
        for i in range(a.steps):
            flush.zero_()                          # L2 flush between timed steps
            step(cfg, q, k, v, do, evs[i])
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ph = [[e[j].elapsed_time(e[j + 1]) for e in evs] for j in range(3)]
    ms_sel, ms_fwd, ms_bwd = (statistics.mean(x) for x in ph)
    ms_step = ms_sel + ms_fwd + ms_bwd
    vals = torch.tensor([ms_step, ms_sel, ms_fwd, ms_bwd], device=dev)
    if dist:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_step, ms_sel, ms_fwd, ms_bwd = vals.tolist()

    e2e_ms, h2d, d2h = e2e_run(cfg, heads, q, k, v, do, max(4, a.steps), 2)
    ev = torch.tensor([e2e_ms], device=dev)
    if dist:
        dist.all_reduce(ev, op=dist.ReduceOp.MAX)
    e2e_ms = ev.item()

    if rank == 0:
        hbm, tf_burst, tf_sus, src = load_peaks()
        f_fwd, f_bwd, f_sel = flops(cfg, heads)
        tokens = cfg["B"] * cfg["N"]
        phases = {}
        for name, ms, fl in (("select", ms_sel, f_sel), ("attn_fwd", ms_fwd, f_fwd),
                             ("attn_bwd", ms_bwd, f_bwd)):
            phases[name] = {"ms": round(ms, 4), "tflops": round(fl / ms / 1e9, 1),
                            "frac_tensor": round(fl / ms / 1e9 / tf_sus, 4)}
        dom = max(phases, key=lambda n: phases[n]["ms"])
        dom_fl = {"select": f_sel, "attn_fwd": f_fwd, "attn_bwd": f_bwd}[dom]
        achieved = dom_fl / (phases[dom]["ms"] * 1e-3) / 1e12
        # a phase of a few ms runs at full clocks: the burst figure is its peak
        peak, peak_name = (tf_burst, "bf16_tflops") if phases[dom]["ms"] < 10 else \
            (tf_sus, "bf16_tflops_sustained")
        for name in phases:
            phases[name]["frac_tensor"] = round(phases[name]["tflops"] / peak, 4)
        line = {
            "metric": METRIC, "value": round(tokens / (ms_step * 1e-3), 1), "unit": UNIT,
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1), seeded",
            "config": config_dict(cfg, world),
            "roofline": {"kernel": dom, "bound": "tensor", "achieved": round(achieved, 2),
                         "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "peak_source": "%s %s (phase of %.2f ms: %s)" % (
                             src, peak_name, phases[dom]["ms"],
                             "burst figure, under 10 ms" if peak_name == "bf16_tflops"
                             else "sustained figure"),
                         "traffic": TRAFFIC_262K.get(dom) if cfg["N"] == 262144 else None,
                         "traffic_source": ("ncu dram__bytes_read+write summed over the phase's "
                                            "kernels, one launch-list capture of this bench at "
                                            "revision %s" % TRAFFIC_REV) if TRAFFIC_REV else
                                           "not captured for this revision"},
            "phases": phases,
            "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": UNIT,
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world},
            "gpu_launches": nlaunch * a.steps,
            "launches_per_step": nlaunch,
            "clocks": clk.summary(),
        }
    del q, k, v, do
    torch.cuda.empty_cache()
    extra = {}
    if not a.no_qsharded:
        extra["qsharded_262k"] = run_qsharded(a, dist, world, rank, dev, flush)
    if not a.no_long:
        extra["long_fwd"] = run_long_fwd(a, dist, world, rank, dev, flush)
    if rank == 0:
        line.update(extra)
        if world == 1 and not a.no_cpu:
            line["cpu_baseline"] = cpu_baseline(cfg, a.cpu_sample)
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def _phase_loop(fn, nph, steps, warmup, flush, dist, dev):
    """Runs fn(events) warmup + steps times (fn records nph + 1 events), flushing L2
    before every timed step; returns the mean ms per phase, max over ranks."""
    for _ in range(warmup):
        fn(None)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nph + 1)] for _ in range(steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        flush.zero_()
        fn(evs[i])
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = [statistics.mean(e[j].elapsed_time(e[j + 1]) for e in evs) for j in range(nph)]
    vals = torch.tensor([sum(ms)] + ms, device=dev)
    if dist:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    return vals.tolist()


def run_qsharded(a, dist, world, rank, dev, flush):
    """The north-star step with the sequence split by query blocks (the layout of
    sequence-parallel training): rank r holds the Q, K, V, dO rows of its
    contiguous query blocks.  One step = NCCL all-gather of K, V + selection
    (pooled-summary all-gathers, equal-area selection rows, row exchange) +
    forward over the local query blocks + backward + the fp32 reduce-scatter of
    the dK/dV partials.  Same total work at every N (strong scaling)."""
    import sharded
    import _bsa
    B, H, N, D, bs, topk = 1, 8, a.n, 64, 64, 16
    if N % (world * bs):
        return {"skipped": "N not divisible by world * block"}
    Ls = N // world
    g = torch.Generator(device=dev).manual_seed(900 + rank)
    q, k, v, do = (torch.randn(B, H, Ls, D, generator=g, device=dev).to(torch.bfloat16)
                   for _ in range(4))
    m = sharded.ShardedBlockSparse(bs=bs, topk=topk, causal=True)
    a0 = rank * (Ls // bs)

    def fn(ev):
        if ev:
            ev[0].record()
        kf, vf, sel = m.select_and_gather(q, k, v)
        if ev:
            ev[1].record()
        o, lse = _bsa.attn_fwd(q, kf, vf, sel, None, bs=bs, causal=True, q_blk0=a0)
        if ev:
            ev[2].record()
        m.backward(q, o, do, (kf, vf, sel, lse))
        if ev:
            ev[3].record()
    ms, ms_sel, ms_fwd, ms_bwd = _phase_loop(fn, 3, a.steps_sub, max(3, a.warmup // 2), flush, dist,
                                             dev)
    return {"N": N, "ms_per_step": round(ms, 4), "tokens_per_s": round(B * N / (ms * 1e-3), 1),
            "phases_ms_max_over_ranks": {"gather_kv+select": round(ms_sel, 4),
                                         "attn_fwd": round(ms_fwd, 4),
                                         "attn_bwd+reduce_scatter": round(ms_bwd, 4)},
            "parallelism": "query blocks sharded %d/rank (NCCL all-gather K, V, pooled summaries, "
                           "selection rows; reduce-scatter dK/dV fp32)" % (N // bs // world),
            "scaling": "strong", "steps": a.steps_sub}


def run_long_fwd(a, dist, world, rank, dev, flush):
    """BASELINE config 3b at N = --long-n (16M by default): forward only, block 128,
    top-16 + own, query blocks sharded over the ranks (one NCCL all-gather of K and
    V, all-gathers of the pooled summaries and of the selection rows), the causal
    top-k streamed through the tensor-core selector so that no nblk x nblk score
    matrix is ever stored; the K/V all-gather (2 (N-1)/N of 34 GB arrives at
    every rank) runs while the selection is computed.  Same total work at every
    N (strong scaling)."""
    import sharded
    import _bsa
    B, H, N, D, bs, topk = 1, 8, a.long_n, 64, 128, 16
    if N % (world * bs):
        return {"skipped": "N not divisible by world * block"}
    Ls = N // world
    nblk = N // bs
    g = torch.Generator(device=dev).manual_seed(700 + rank)
    q, k, v = (torch.randn(B, H, Ls, D, generator=g, device=dev).to(torch.bfloat16)
               for _ in range(3))
    m = sharded.ShardedBlockSparse(bs=bs, topk=topk, causal=True)
    a0 = rank * (Ls // bs)
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated(dev)
    torch.cuda.reset_peak_memory_stats(dev)

    kv_group = dist.new_group(list(range(world))) if dist else None

    def fn(ev):
        if ev:
            ev[0].record()
        m.forward_pipelined(q, k, v, kv_group=kv_group)
        if ev:
            ev[1].record()
    ms, = _phase_loop(fn, 1, a.steps_long, 3, flush, dist, dev)[1:]
    # the phases on their own (not overlapped), for the record
    def fn2(ev):
        if ev:
            ev[0].record()
        kf, vf, sel = m.select_and_gather(q, k, v)
        if ev:
            ev[1].record()
        _bsa.attn_fwd(q, kf, vf, sel, None, bs=bs, causal=True, want_lse=False, q_blk0=a0)
        if ev:
            ev[2].record()
    _, ms_kvsel, ms_fwd = _phase_loop(fn2, 2, max(2, a.steps_long // 2), 1, flush, dist, dev)
    peak = torch.cuda.max_memory_allocated(dev) - base
    fwd_flops = 4.0 * B * H * N * (topk + 1) * bs * D
    score_bytes = 4.0 * nblk * nblk * H / world
    return {"N": N, "ms_per_step": round(ms, 3), "tokens_per_s": round(B * N / (ms * 1e-3), 1),
            "phases_ms_max_over_ranks": {
                "unpipelined: select+gather_kv (overlapped)": round(ms_kvsel, 3),
                "unpipelined: attn_fwd": round(ms_fwd, 3)},
            "pipelining": "K/V gathered per head on a second communicator while the selection "
                          "runs; head h's attention starts when its K/V have arrived",
            "gather_bytes_per_rank": int(2 * (world - 1) * q.numel() * 2),
            "attn_fwd_tflops_per_gpu": round(fwd_flops / world / (ms_fwd * 1e-3) / 1e12, 1),
            "peak_extra_alloc_bytes_per_rank": int(peak),
            "score_matrix_bytes_per_rank_if_stored": int(score_bytes),
            "score_matrix_stored": bool(peak >= score_bytes),
            "parallelism": "query blocks sharded %d/rank" % (nblk // world),
            "config": "B1 H8 D64 block128 top16 (+own) causal bf16, forward only",
            "scaling": "strong", "steps": a.steps_long}


# ---------------------------------------------------------------- CPU baseline
class CpuSample:
    """The reference's CPU gather path (restated in oracle/, fp32, all host threads)
    on a bounded sample: S query blocks [nblk-S, nblk) of every head, with the
    reference's own selection algorithm for those rows (score against every key
    block, mask, top-k: src/ssa_model.py:151-162) and the gather attention forward
    + autograd backward (src/ssa_model.py:57-90).  Cost per query block is
    independent of its position, so tokens/s = S*bs / sample time."""

    def __init__(self, cfg, heads, S):
        from oracle import oracle as O
        S = min(S, cfg["nblk"] - 1)
        self.O = O
        torch.set_num_threads(os.cpu_count() or 1)
        self.cfg, self.heads, self.S = cfg, heads, S
        B, N, D = cfg["B"], cfg["N"], cfg["D"]
        g = torch.Generator().manual_seed(7)
        self.q, self.k, self.v, self.do = (
            torch.randn(B, heads, N, D, generator=g).to(torch.bfloat16).float() for _ in range(4))

    def run(self):
        cfg, S = self.cfg, self.S
        bs, nblk = cfg["bs"], cfg["nblk"]
        i0 = nblk - S
        B, H, N, D = self.q.shape
        t0 = time.perf_counter()
        qp = self.q[:, :, i0 * bs:].reshape(B, H, S, bs, D).mean(3)
        kp = self.k.reshape(B, H, nblk, bs, D).mean(3)
        raw = qp @ kp.transpose(-1, -2)                          # (B,H,S,nblk)
        rows = torch.arange(i0, nblk).view(S, 1)
        cols = torch.arange(nblk).view(1, nblk)
        raw = raw.masked_fill((cols >= rows), float("-inf"))     # exclude own + future
        top = raw.topk(cfg["topk"], dim=-1).indices
        own = rows.view(1, 1, S, 1).expand(B, H, S, 1)
        sel_rows = torch.cat([own, top], -1)
        sel = torch.zeros(B, H, nblk, cfg["kk"], dtype=torch.long)
        sel[:, :, i0:] = sel_rows
        for c0 in range(i0, nblk, 128):     # bounded memory: 128 query blocks at a time
            self.O.attention_grads(self.q, self.k, self.v, sel, self.do, None, bs=bs, causal=True,
                                   dtype=torch.float32, qblk_range=(c0, min(c0 + 128, nblk)))
        return time.perf_counter() - t0

    def tokens(self):
        return self.cfg["B"] * self.S * self.cfg["bs"]


def cpu_baseline(cfg, S):
    smp = CpuSample(cfg, cfg["H"], S)
    smp.run()                                                     # warm-up
    t = smp.run()
    return {"value": round(smp.tokens() / t, 1), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": "query blocks %d..%d of all %d heads at N=%d (%d tokens), selection + gather "
                      "fwd + autograd bwd in fp32, %.2f s" % (cfg["nblk"] - S, cfg["nblk"], cfg["H"],
                                                               cfg["N"], smp.tokens(), t)}


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = workload(a)
    smp = CpuSample(cfg, cfg["H"], a.ref_sample)
    for _ in range(a.warmup):
        smp.run()
    ts = [smp.run() for _ in range(a.steps)]
    t = statistics.mean(ts)
    value = smp.tokens() / t
    cores = torch.get_num_threads()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    frac = smp.S / cfg["nblk"]
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": UNIT,
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(t * 1e3, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32 (bf16-rounded inputs)",
        "data": "synthetic N(0,1), seeded",
        "config": config_dict(cfg, world),
        "sample_fraction": round(frac, 6),
        "sample": "each step = the last %d of %d query blocks of all %d heads (%d tokens) through "
                  "selection + gather fwd + autograd bwd; ms_per_step is that sample's measured "
                  "time, value = its tokens / time (the per-block cost does not depend on the "
                  "position)" % (smp.S, cfg["nblk"], cfg["H"], smp.tokens()),
        "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": "%d query blocks x %d heads per step (%d tokens), mean of %d "
                                   "steps" % (smp.S, cfg["H"], smp.tokens(), a.steps)},
        "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- other configurations
def _timed(fn, steps, warmup, flush, dev_index, phases=1):
    """Runs fn(events) `steps` times after `warmup` untimed runs, flushing L2
    before each timed run; fn records phases+1 events.  Returns (mean ms per
    phase, clock summary)."""
    for _ in range(warmup):
        fn(None)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(phases + 1)] for _ in range(steps)]
    with ClockSampler(dev_index, enabled=int(os.environ.get("RANK", "0")) == 0) as clk:
        for i in range(steps):
            flush.zero_()
            fn(evs[i])
        torch.cuda.synchronize()
    ms = [statistics.mean(e[j].elapsed_time(e[j + 1]) for e in evs) for j in range(phases)]
    return ms, clk.summary()


def _line(metric, value, unit, ms, a, world, scaling, dtype, config, roofline, clocks, extra=None):
    d = {"metric": metric, "value": round(value, 1), "unit": unit, "n_gpus": world, "steps": a.steps,
         "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
         "scaling": scaling, "vs_baseline": None, "dtype": dtype, "data": "synthetic N(0,1), seeded",
         "config": config, "roofline": roofline, "clocks": clocks}
    d.update(extra or {})
    print(json.dumps(d), flush=True)


def _roof(name, fl, ms, peak, src):
    """peak: the sustained figure; phases under 10 ms are rated against the burst one."""
    _, tf_burst, _, kind = load_peaks()
    if ms < 10:
        peak, src = tf_burst, "%s bf16_tflops (burst figure: phase of %.2f ms)" % (kind, ms)
    ach = fl / (ms * 1e-3) / 1e12
    return {"kernel": name, "bound": "tensor", "achieved": round(ach, 2), "peak": peak,
            "unit": "TFLOP/s", "frac": round(ach / peak, 4), "peak_source": src, "traffic": None}


def run_config(a):
    """BASELINE configurations 2, 3b, 4, 5 (see the module docstring of each branch)."""
    import _bsa
    import selection
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    hbm, tf_burst, tf_sus, src = load_peaks()
    psrc = "%s bf16_tflops_sustained" % src
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(11 + rank)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(torch.bfloat16)

    if a.config == "2":
        # small-LM training layer: B8 H8 N8192 D64 block 64, gate-coupled top-16 (+own)
        B, H, N, D, bs, topk = 8, 8, 8192, 64, 64, 16
        q, k, v = (rnd(B, H, N, D, scale=0.5) for _ in range(3))
        do = rnd(B, H, N, D)

        def fn(ev):
            if ev:
                ev[0].record()
            sel, gate, _ = selection.select_meanpool(q, k, bs=bs, topk=topk, want_gate=True)
            o, lse = _bsa.attn_fwd(q, k, v, sel, gate, bs=bs, causal=True)
            _bsa.attn_bwd(q, k, v, o, do, sel, lse, gate, bs=bs, causal=True, want_dgate=True)
            if ev:
                ev[1].record()
        (ms,), clk = _timed(fn, a.steps, a.warmup, flush, local)
        fwd = 4.0 * B * H * N * (topk + 1) * bs * D
        if rank == 0:
            _line("layer fwd+bwd tokens/s (B8 H8 N8192, gate-coupled selection)", B * N / (ms * 1e-3),
                  "tokens/s", ms, a, 1, "weak", "bf16",
                  {"workload": "BASELINE config 2: B8 H8 N8192 D64 block64 top16 (+own) causal, "
                               "gate = logsigmoid(selected scores), dgate computed", "B": B, "H": H,
                   "N": N, "l2": "256 MB buffer written between timed steps"},
                  _roof("selection+fwd+bwd", 3.5 * fwd, ms, tf_sus, psrc), clk)
    elif a.config == "3b":
        # long forward: B1 H8 D64 block 128 top-16 (+own), query blocks sharded over the ranks
        import sharded
        B, H, D, bs, topk = 1, 8, 64, 128, 16
        N = a.n
        if N % (world * bs):
            raise SystemExit("N must be a multiple of world * 128")
        Ls = N // world
        q, k, v = (rnd(B, H, Ls, D) for _ in range(3))
        m = sharded.ShardedBlockSparse(bs=bs, topk=topk, causal=True) if dist else None

        def fn(ev):
            if ev:
                ev[0].record()
            if m:
                kf, vf, sel = m.select_and_gather(q, k, v)
                if ev:
                    ev[1].record()
                o, _ = _bsa.attn_fwd(q, kf, vf, sel, bs=bs, causal=True, want_lse=False,
                                     q_blk0=dist.get_rank() * (Ls // bs))
            else:
                sel, _, _ = selection.select_meanpool(q, k, bs=bs, topk=topk)
                if ev:
                    ev[1].record()
                o, _ = _bsa.attn_fwd(q, k, v, sel, bs=bs, causal=True, want_lse=False)
            if ev:
                ev[2].record()
        if dist:
            dist.barrier()
        (ms_sel, ms_fwd), clk = _timed(fn, a.steps, a.warmup, flush, local, phases=2)
        vals = torch.tensor([ms_sel + ms_fwd, ms_sel, ms_fwd], device=dev)
        if dist:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        ms, ms_sel, ms_fwd = vals.tolist()
        fwd = 4.0 * B * H * Ls * (topk + 1) * bs * D
        if rank == 0:
            _line("long-context fwd tokens/s at N=%d (selection + all-gather + forward)" % N,
                  B * N / (ms * 1e-3), "tokens/s", ms, a, world, "strong", "bf16",
                  {"workload": "BASELINE config 3b: forward only, B1 H8 N%d D64 block128 top16 "
                               "(+own) causal, streaming top-k (no nblk^2 scores)" % N,
                   "N": N, "parallelism": "query blocks sharded %d/rank, NCCL all-gather of K, V and "
                                          "pooled keys" % (N // bs // world) if dist else "none",
                   "l2": "256 MB buffer written between timed steps"},
                  _roof("attn_fwd", fwd, ms_fwd, tf_sus, psrc), clk,
                  {"phases": {"gather_kv+select" if dist else "select": round(ms_sel, 3),
                              "attn_fwd": round(ms_fwd, 3)}})
    elif a.config == "4":
        # Qwen GQA prefill: N65536 Hq16 Hkv2 D256 block 128, partial RoPE (64 dims, theta 1e7),
        # SelectMax top-32 + own + sink, sigmoid output gate; also the all-blocks (dense) mode
        import qwen_blocksparse as qb
        B, Hq, Hkv, N, D, bs = 1, 16, 2, 65536, 256, 128
        q = rnd(B, Hq, N, D)
        k, v = rnd(B, Hkv, N, D), rnd(B, Hkv, N, D)
        gate = rnd(B, N, Hq * D)
        cos, sin = qb.rope_cos_sin(N, 64, 1e7, torch.bfloat16, dev)
        sm = qb.SelectMax(32, bs)
        out = {}
        for mode, sel in (("select", sm), ("all_blocks", qb.SelectAll(bs))):
            def fn(ev, sel=sel):
                if ev:
                    ev[0].record()
                qb.qwen_attention(q, k, v, cos, sin, gate, selector=sel, topk=32, bs=bs)
                if ev:
                    ev[1].record()
            (ms,), clk = _timed(fn, a.steps, a.warmup, flush, local)
            out[mode] = (ms, clk)
        ms, clk = out["select"]
        kk = 34
        fwd = 4.0 * B * Hq * N * kk * bs * D
        dense = 2.0 * B * Hq * N * N * D      # causal dense: half of 4*N*N*D
        if rank == 0:
            _line("Qwen GQA prefill tokens/s (N65536 Hq16 Hkv2 D256, SelectMax top-32)",
                  B * N / (ms * 1e-3), "tokens/s", ms, a, 1, "weak", "bf16",
                  {"workload": "BASELINE config 4: RoPE(64 of 256 dims, theta 1e7) + SelectMax "
                               "top32 + own + sink (width 34) + GQA attention + sigmoid gate",
                   "N": N, "l2": "256 MB buffer written between timed steps"},
                  _roof("rope+select+attn_fwd", fwd, ms, tf_sus, psrc), clk,
                  {"all_blocks": {"ms": round(out["all_blocks"][0], 3),
                                  "tokens_per_s": round(B * N / (out["all_blocks"][0] * 1e-3), 1),
                                  "tflops": round(dense / out["all_blocks"][0] / 1e9, 1)}})
    elif a.config == "5":
        # LSH selector: B1 H8 N131072 D64 block 64, 4 sign planes x 4 rounds, cap 16, top-16
        B, H, N, D, bs = 1, 8, 131072, 64, 64
        q, k, v = (rnd(B, H, N, D) for _ in range(3))
        planes = selection.lsh_planes(D, 4, 4, 0).to(dev)

        def fn(ev):
            if ev:
                ev[0].record()
            sel, _, _ = selection.select_lsh(q, k, bs=bs, topk=16, n_rounds=4, n_planes=4, cap=16,
                                             planes=planes)
            if ev:
                ev[1].record()
            _bsa.attn_fwd(q, k, v, sel, bs=bs, causal=True, want_lse=False)
            if ev:
                ev[2].record()
        (ms_sel, ms_fwd), clk = _timed(fn, a.steps, a.warmup, flush, local, phases=2)
        ms = ms_sel + ms_fwd
        fwd = 4.0 * B * H * N * 17 * bs * D
        if rank == 0:
            _line("LSH-selected fwd tokens/s (N131072 H8, hash+bucket+candidates+read)",
                  B * N / (ms * 1e-3), "tokens/s", ms, a, 1, "weak", "bf16",
                  {"workload": "BASELINE config 5: B1 H8 N131072 D64 block64, pooled+normalised "
                               "blocks, sign of 4 hyperplanes x 4 rounds, cap 16, top-16 (+own)",
                   "N": N, "l2": "256 MB buffer written between timed steps"},
                  _roof("attn_fwd", fwd, ms_fwd, tf_sus, psrc), clk,
                  {"phases": {"lsh_select(pool+hash+bucket+select)": round(ms_sel, 3),
                              "attn_fwd": round(ms_fwd, 3)}})
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seqlen", "--n", dest="n", type=int, default=262144,
                    help="sequence length (default 262144; 1048576 for --config 3b)")
    ap.add_argument("--cpu-sample", type=int, default=2048,
                    help="query blocks in the cpu_baseline sample (about 10 s of CPU work)")
    ap.add_argument("--ref-sample", type=int, default=256,
                    help="query blocks per step of the --impl reference arm")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-long", action="store_true", help="skip the long_fwd (16M) sub-object")
    ap.add_argument("--kernels-only", action="store_true",
                    help="run warm-up + steps of the hot path only (for ncu captures); no JSON line")
    ap.add_argument("--no-qsharded", action="store_true", help="skip the qsharded_262k sub-object")
    ap.add_argument("--long-n", type=int, default=1 << 24, help="tokens of the long_fwd sub-object")
    ap.add_argument("--steps-long", type=int, default=5, help="timed steps of long_fwd")
    ap.add_argument("--steps-sub", type=int, default=10, help="timed steps of qsharded_262k")
    ap.add_argument("--config", default="3a", choices=["3a", "2", "3b", "4", "5"],
                    help="BASELINE configuration (3a = the driver line)")
    a = ap.parse_args()
    if a.warmup < 3:
        a.warmup = 3
    if a.impl == "reference":
        run_reference(a)
    elif a.config != "3a":
        if a.config == "3b" and a.n == 262144:
            a.n = 1 << 20
        run_config(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
