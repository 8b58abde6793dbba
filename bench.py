"""Benchmark of the fused diffusion stencil (one JSON line on rank 0).

Workload (default, "fused_fwd"): the single-GPU fused forward of the stencil
on bf16 x[B=1, L, D=512] ~ N(0,1), alpha = 0.1, `--stencil-steps` steps in ONE
launch ([B, L, D] layout, the model / serving layout).  One bench step = one
fused call over one batch.  Inputs and outputs rotate through a pool of
buffers larger than L2, so every call streams from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--L 65536] [--stencil-steps 4] [--no-sweep]

N > 1 (torchrun, one rank per GPU): every rank runs the same per-GPU workload
on its own GPU (independent replicas, weak scaling; the stencil of one
sequence shards only with the L-sharded workload, `--workload sharded`).

Reported: `value` tokens/s with inputs resident in HBM (device-timed with CUDA
events over CUDA-graph replays of the calls, max over ranks); `e2e` the same
through the public API, called eagerly, with pinned host buffers
(H2D + kernel + D2H each step); `roofline` of the fused kernel against the
measured HBM copy bandwidth; `cpu_baseline` the CPU oracle (the reference's
algorithm in PyTorch) on the host cores; `clocks` sampled during timing.
`--impl reference` times that CPU implementation alone.
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

REPO = Path(__file__).resolve().parent
for _p in (str(REPO), str(REPO / "continuous-time-attention_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

REF_DIR = REPO / "baseline" / "_ref"  # the unmodified reference install
METRIC = "fused diffusion stencil tokens/s & HBM GB/s (% of peak) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:  # noqa: BLE001
            pass
    return FALLBACK_HBM_GBS, "fallback"


def _ncu_traffic(key: str):
    p = REPO / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    try:
        entry = json.loads(p.read_text()).get(key)
        return None if entry is None else entry.get("per_launch_bytes")
    except Exception:  # noqa: BLE001
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [v.strip() for v in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU side: the oracle (the reference's algorithm) on the host cores
# ---------------------------------------------------------------------------
def _cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _cpu_impl():
    """The CPU implementation the CPU arm times: the reference's own
    `_diffusion_steps_bld` (src/cta/serving_vllm.py:29-46) from the unmodified
    install under baseline/_ref ("reference"), else the oracle's restatement of
    it in torch fp32 ("port").  Returns (fn(x, steps), kind, description)."""
    if (REF_DIR / "cta" / "serving_vllm.py").is_file():
        if str(REF_DIR) not in sys.path:
            sys.path.append(str(REF_DIR))
        try:
            from cta.serving_vllm import _diffusion_steps_bld as ref_fn

            return (lambda x, steps: ref_fn(x, alpha=0.1, steps=steps), "reference",
                    "the reference's own _diffusion_steps_bld (PyTorch CPU, unmodified, from baseline/_ref)")
        except Exception:  # noqa: BLE001 - fall back to the port below
            pass
    from oracle import diffusion_oracle as O

    return (lambda x, steps: O.steps_bld(x, alpha=0.1, steps=steps), "port",
            "the CPU oracle (the reference's _diffusion_steps_bld restated in torch fp32)")


def cpu_oracle_times(L: int, D: int, steps: int, timed: int, warmup: int = 2):
    """Seconds per call of the CPU implementation (`_cpu_impl`) on the FULL bf16
    [1, L, D] tensor, all host threads, after `warmup` untimed calls."""
    fn, _, _ = _cpu_impl()
    torch.set_num_threads(os.cpu_count() or 1)
    torch.manual_seed(0)
    x = torch.randn(1, L, D).to(torch.bfloat16)
    for _ in range(warmup):
        fn(x, steps)
    times = []
    for _ in range(timed):
        t0 = time.perf_counter()
        fn(x, steps)
        times.append(time.perf_counter() - t0)
    return times


def _cpu_line(L: int, D: int, steps: int, times) -> dict:
    _, kind, desc = _cpu_impl()
    p50 = statistics.median(times)
    return {
        "value": L / p50,
        "unit": "tokens/s",
        "cores": torch.get_num_threads(),
        "cpu_model": _cpu_model(),
        "kind": kind,
        "p50_ms": p50 * 1e3,
        "sample": f"p50 of {len(times)} calls (after 2 warm-ups) of {desc} on the full bf16 [1, {L}, {D}] "
                  f"tensor, steps {steps}",
    }


def cpu_reference_rate(L: int, D: int, steps: int):
    """cpu_baseline of the GPU arm: the same measurement as `--impl reference`."""
    return _cpu_line(L, D, steps, cpu_oracle_times(L, D, steps, timed=10))


def run_reference(args, rank: int) -> None:
    """The reference arm: the reference's CPU implementation of the path on the
    host cores -- its own `_diffusion_steps_bld` from baseline/_ref when that
    install exists, else the oracle port (`_cpu_impl`).  One step = one call over
    the full [1, L, D] input; value = tokens / p50 step."""
    if rank != 0:
        return
    L, D, S = args.L, args.D, args.stencil_steps
    times = cpu_oracle_times(L, D, S, timed=max(args.steps, 1), warmup=max(2, min(args.warmup, 5)))
    cpu = _cpu_line(L, D, S, times)
    v = cpu["value"]
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": len(times), "warmup": max(2, min(args.warmup, 5)), "ms_per_step": cpu["p50_ms"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _config(args),
        "cpu_baseline": cpu,
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


CALLS_PER_STEP = 256


def _config(args):
    return {"workload": "fused_fwd_bld", "B": 1, "L": args.L, "D": args.D, "steps": args.stencil_steps,
            "alpha": 0.1, "layout": "bld", "global_batch": args.gpus, "seq_len": args.L,
            "calls_per_step": CALLS_PER_STEP,
            "parallelism": f"replicas x{args.gpus}",
            "l2": "rotating input/output buffers, >= 4x L2 per rank"}


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
def _time_launches(fn, n: int, stream) -> float:
    """Seconds for n eager calls, CUDA events on the launching stream."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(n):
        fn(i)
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / 1e3


class GraphLoop:
    """`per_graph` consecutive calls captured once as a CUDA graph; timing replays
    it, so the device runs the launches back to back without host gaps."""

    def __init__(self, fn, per_graph: int):
        self.per_graph = per_graph
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(per_graph):  # warm every buffer / attribute outside capture
                fn(i)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            for i in range(per_graph):
                fn(i)
        torch.cuda.synchronize()

    def time_replays(self, reps: int, stream) -> float:
        """Seconds for exactly `reps` replays (CUDA events on the launching stream)."""
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(reps):
            self.graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / 1e3

    def time(self, n_calls: int, stream) -> tuple[float, int]:
        reps = max(1, (n_calls + self.per_graph - 1) // self.per_graph)
        return self.time_replays(reps, stream), reps * self.per_graph


def _check_windows(x: torch.Tensor, y: torch.Tensor, steps: int, contracted: bool) -> list:
    """Compare output windows at both ends and the middle of a [1, L, D] result
    with the CPU oracle run on the matching input windows, in the arithmetic the
    call used (bit-exact)."""
    from oracle import diffusion_oracle as O

    L = x.shape[1]
    w = min(512, L)
    bad = []
    for a in sorted({0, max(0, L // 2 - w // 2), L - w}):
        b = min(L, a + w)
        ws, we = max(0, a - 2 * steps), min(L, b + 2 * steps)
        ref = O.window_bld(x[:, ws:we].cpu(), win_start=ws, global_len=L, out_start=a, out_stop=b, alpha=0.1,
                           steps=steps, contracted=contracted)
        if not torch.equal(ref, y[:, a:b].cpu()):
            bad.append((a, b))
    return bad


def _eager_host(dev) -> dict:
    """Host cost per eager call (Python validation + ctypes + launch) of the layer
    and the mixer at bf16 [1, 4096, 512], and the wall time per call with the
    device in the loop; no CUDA graphs."""
    from types import SimpleNamespace

    from cta_b200.pde_layers import DiffusionPDELayer
    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer

    x = torch.randn(1, 4096, 512, device=dev, dtype=torch.bfloat16)
    layer = DiffusionPDELayer(512, layout="bld").to(dev)
    mixer = CtaPostAttnMixer(CtaConfig(steps=4, alpha=0.1, trace=False))
    flat = x[0]
    md = SimpleNamespace(max_query_len=4096, query_start_loc=torch.tensor([0, 2048, 4096], dtype=torch.int32,
                                                                           device=dev), num_actual_tokens=4096)
    calls = {
        "pde_layer_fwd": lambda: layer(x),
        "mixer_dense": lambda: mixer(x),
        "mixer_packed": lambda: mixer(flat, attn_metadata=md),
        "ops_bld_forward": None,
    }
    from cta_b200 import ops

    calls["ops_bld_forward"] = lambda: ops.bld_forward(x, [0.1] * 4, 4)
    out = {}
    with torch.no_grad():
        for name, fn in calls.items():
            for _ in range(20):
                fn()
            torch.cuda.synchronize()
            n = 400
            t0 = time.perf_counter()
            for _ in range(n):
                fn()
            t1 = time.perf_counter()
            torch.cuda.synchronize()
            t2 = time.perf_counter()
            out[name] = {"host_us": round((t1 - t0) / n * 1e6, 2), "wall_us": round((t2 - t0) / n * 1e6, 2)}
    return out


def reference_gpu_modules():
    """The reference's own GPU path, unmodified, from baseline/_ref (placed there
    by baseline/install_reference.py): (kernels.diffusion_triton,
    cta.serving_vllm) and None, or None and the reason it is unavailable."""
    if not (REF_DIR / "kernels" / "diffusion_triton.py").is_file():
        return None, "no reference install under baseline/_ref (python baseline/install_reference.py --ref <root>)"
    if str(REF_DIR) not in sys.path:
        sys.path.append(str(REF_DIR))
    try:
        import cta.serving_vllm as sv
        import kernels.diffusion_triton as kt
    except Exception as e:  # noqa: BLE001 - reported, not raised
        return None, f"reference import failed: {type(e).__name__}: {e}"
    if getattr(kt, "triton", None) is None:
        return None, "triton is not importable"
    return (kt, sv), None


def _time_eager(fn, n: int, warmup: int, stream) -> float:
    """Seconds per eager call (host work included), CUDA events on `stream`."""
    for i in range(warmup):
        fn(i)
    return _time_launches(fn, n, stream) / n


def _reference_gpu(dev, full: bool) -> dict:
    """The reference's GPU path timed beside ours on this GPU, both called
    eagerly through their public APIs on the same inputs (rotating buffers
    larger than L2), with a bit-for-bit comparison of the outputs:

      * the vLLM post-attention mixer on bf16 [1, 65536, 512], steps 4: the
        reference transposes to [B, D, L], runs its fused Triton s4 kernel and
        transposes back (src/cta/serving_vllm.py:195-266); ours is one
        [B, L, D] launch;
      * the kernel API diffusion_triton_fused on bf16 [1, 512, 65536]
        (kernels/diffusion_triton.py:829-868, 891-910), steps 4 (2, 4, 8 with
        `full`);
      * with `full`, the packed prefill of 64 sequences U[512, 8192] x 4096
        bf16 (src/cta/serving_vllm.py:72-111, 275-303) under the reference rule.
    """
    mods, why = reference_gpu_modules()
    if mods is None:
        return {"unavailable": why}
    kt, sv = mods
    from cta_b200 import diffusion as our_kernels
    from cta_b200 import serving_vllm as our_sv

    stream = torch.cuda.current_stream(dev)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    out = {"source": "baseline/_ref (the reference tree, unmodified; its Triton kernels JIT-compiled here)",
           "timing": "eager calls through each public API, CUDA events, rotating inputs > L2", "rows": []}

    def row(name, ref_fn, our_fn, tokens, calls=20, steps=None):
        yr, yo = ref_fn(0), our_fn(0)
        # elements that differ, and by how many units in the last place (bf16)
        d = (yr.view(torch.int16).int() - yo.view(torch.int16).int()).abs()
        kern = {2: kt._diffusion_fused_s2_kernel, 4: kt._diffusion_fused_s4_kernel,
                8: kt._diffusion_fused_s8_kernel}.get(steps)
        best = getattr(kern, "best_config", None) if kern is not None else None
        t_ref = _time_eager(ref_fn, calls, 3, stream)
        t_our = _time_eager(our_fn, calls, 3, stream)
        out["rows"].append({"workload": name, "reference_us": round(t_ref * 1e6, 1), "ours_us": round(t_our * 1e6, 1),
                            "speedup": round(t_ref / t_our, 2), "reference_tokens/s": round(tokens / t_ref),
                            "ours_tokens/s": round(tokens / t_our), "bit_identical": bool(int(d.max()) == 0),
                            "elements_differing": int((d > 0).sum()), "max_ulp": int(d.max()),
                            "reference_config": None if best is None else f"BLOCK {best.kwargs.get('BLOCK')}"})

    L, D, S = 65536, 512, 4
    nb = max(2, (4 * l2) // (L * D * 2) + 1)
    gen = torch.Generator(device=dev).manual_seed(77)
    xs = [torch.randn(1, L, D, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(nb)]
    ref_mixer = sv.CtaPostAttnMixer(sv.CtaConfig(steps=S, alpha=0.1, trace=False))
    our_mixer = our_sv.CtaPostAttnMixer(our_sv.CtaConfig(steps=S, alpha=0.1, trace=False))
    row(f"mixer bf16 [1, {L}, {D}] steps {S}", lambda i: ref_mixer(xs[i % nb], is_prefill=True),
        lambda i: our_mixer(xs[i % nb], is_prefill=True), L, steps=S)
    xt = [x.view(1, D, L) for x in xs]  # the same bytes read as [B, D, L]
    for s in ((2, 4, 8) if full else (4,)):
        row(f"diffusion_triton_fused bf16 [1, {D}, {L}] steps {s}",
            lambda i, s=s: kt.diffusion_triton_fused(xt[i % nb], alpha=0.1, steps=s),
            lambda i, s=s: our_kernels.diffusion_triton_fused(xt[i % nb], alpha=0.1, steps=s), L, steps=s)
    del xs, xt
    if full:
        g = torch.Generator().manual_seed(0)
        lens = torch.randint(512, 8193, (64,), generator=g)
        qsl = torch.zeros(65, dtype=torch.int32)
        qsl[1:] = torch.cumsum(lens, 0)
        T, Dv = int(qsl[-1]), 4096
        xv = [torch.randn(T, Dv, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(2)]
        from types import SimpleNamespace
        md = SimpleNamespace(query_start_loc=qsl.to(dev), max_query_len=int(lens.max()))
        row(f"packed prefill 64 seqs U[512, 8192] x {Dv} bf16 steps {S} (reference rule)",
            lambda i: ref_mixer(xv[i % 2], attn_metadata=md, is_prefill=True),
            lambda i: our_mixer(xv[i % 2], attn_metadata=md, is_prefill=True), T, calls=5, steps=S)
        del xv
    torch.cuda.empty_cache()
    return out


def _sharded_parts(args, rank: int, world: int, dev) -> dict:
    """C5 on the ranks of this job: bf16 x[1, 1048576, 4096], steps 8, split evenly
    along L (strong scaling), forward + adjoint per step with the NCCL halo
    exchange; per-part device times from a separately timed pass; windows at the
    shard edges and the global ends checked against the oracle."""
    import torch.distributed as dist

    from cta_b200.sharded import even_shards, sharded_diffusion

    L, D, S = 1 << 20, 4096, 8
    spec = even_shards(L, world, rank)
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(1, spec.local_len, D, device=dev, dtype=torch.bfloat16, generator=gen)
    g = torch.randn(1, spec.local_len, D, device=dev, dtype=torch.bfloat16, generator=gen)
    comm = torch.cuda.Stream(device=dev, priority=-1)
    stream = torch.cuda.current_stream(dev)
    overlap = args.shard_exchange == "overlap"

    def step(timing=None):
        y = sharded_diffusion(x, spec, alpha=0.1, steps=S, comm_stream=comm, timing=timing, overlap=overlap)
        dx = sharded_diffusion(g, spec, alpha=0.1, steps=S, backward=True, comm_stream=comm, timing=timing,
                               overlap=overlap)
        return y, dx

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    k = 10
    t = _max_over_ranks(_time_launches(lambda i: step(), k, stream), dev, world) / k
    # per-part device times (events add no work; a separate pass so the headline has none)
    parts = {}
    for _ in range(3):
        tm = {}
        step(tm)
        torch.cuda.synchronize()
        for key, evs in tm.items():
            parts.setdefault(key, []).append(sum(a.elapsed_time(b) for a, b in evs))
    parts = {k: round(statistics.median(v) * 1e3, 1) for k, v in parts.items()}
    # oracle check of the output rows next to this shard's edges
    y, dx = step()
    torch.cuda.synchronize()
    bad = _sharded_check(x, y, spec, S, world)
    del x, g, y, dx
    torch.cuda.empty_cache()
    peak, _ = _peaks()
    bytes_rank = 4 * spec.local_len * D * 2
    nranks = dist.get_world_size() if world > 1 else 1
    return {"workload": "sharded_fwd_adjoint", "L": L, "D": D, "steps": S, "ranks": world,
            "comm_nranks": nranks, "exchange": args.shard_exchange, "scaling": "strong", "ms_per_step": t * 1e3,
            "tokens/s": L / t,
            "hbm_frac_per_gpu": bytes_rank / t / 1e9 / peak, "parts_us": parts,
            "oracle_windows_ok": not bad, "bad_windows": bad[:4]}


def _sharded_check(x, y, spec, S: int, world: int) -> list:
    """Rows [0, 256) and [n-256, n) of this shard against the oracle window over
    the neighbours' S rows (received point-to-point, outside any timing)."""
    import torch.distributed as dist

    from oracle import diffusion_oracle as O

    n = spec.local_len
    lo = hi = None
    if world > 1:
        ops_ = []
        if spec.rank > 0:
            lo = torch.empty_like(x[:, :S])
            ops_ += [dist.P2POp(dist.isend, x[:, :S].contiguous(), spec.rank - 1),
                     dist.P2POp(dist.irecv, lo, spec.rank - 1)]
        if spec.rank + 1 < world:
            hi = torch.empty_like(x[:, :S])
            ops_ += [dist.P2POp(dist.isend, x[:, n - S:].contiguous(), spec.rank + 1),
                     dist.P2POp(dist.irecv, hi, spec.rank + 1)]
        for w in dist.batch_isend_irecv(ops_):
            w.wait()
    w = min(256, n)
    bad = []
    head = torch.cat(([lo] if lo is not None else []) + [x[:, : w + S]], dim=1).cpu()
    hs = spec.pos_offset - (S if lo is not None else 0)
    ref = O.window_bld(head, win_start=hs, global_len=spec.global_len, out_start=spec.pos_offset,
                       out_stop=spec.pos_offset + w, alpha=0.1, steps=S, contracted=True)
    if not torch.equal(ref, y[:, :w].cpu()):
        bad.append(("lo", spec.rank))
    tail = torch.cat([x[:, n - w - S:]] + ([hi] if hi is not None else []), dim=1).cpu()
    ts = spec.pos_offset + n - w - S
    ref = O.window_bld(tail, win_start=ts, global_len=spec.global_len, out_start=spec.pos_offset + n - w,
                       out_stop=spec.pos_offset + n, alpha=0.1, steps=S, contracted=True)
    if not torch.equal(ref, y[:, n - w:].cpu()):
        bad.append(("hi", spec.rank))
    return bad


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch.distributed as dist

    from cta_b200 import _lib, ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L, D, S = args.L, args.D, args.stencil_steps
    esize = 2
    tensor_bytes = L * D * esize
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    nbuf = max(2, min(64, (4 * l2) // tensor_bytes + 1))
    torch.manual_seed(1234 + rank)
    xs = [torch.randn(1, L, D, device=dev, dtype=torch.bfloat16) for _ in range(nbuf)]
    ys = [torch.empty_like(xs[0]) for _ in range(nbuf)]
    alphas = [0.1] * S
    stream = torch.cuda.current_stream(dev)

    def call(i):
        ops.bld_forward(xs[i % nbuf], alphas, S, out=ys[i % nbuf])

    if args.mode == "kernel":
        # bare launches for profilers: no sampler, e2e, sweep or CPU baseline
        for i in range(args.warmup):
            call(i)
        t = _time_launches(call, args.steps, stream)
        if rank == 0:
            print(json.dumps({"mode": "kernel", "launches": args.steps, "us_per_call": t / args.steps * 1e6,
                              "config": _config(args)}), flush=True)
        return
    # one bench step = CALLS_PER_STEP consecutive calls (one CUDA-graph replay)
    loop = GraphLoop(call, CALLS_PER_STEP)
    for _ in range(args.warmup):
        loop.graph.replay()
    torch.cuda.synchronize()
    bad = _check_windows(xs[0], ys[0], S, contracted=True)  # the last replay wrote ys[0] from xs[0]
    if bad:
        raise RuntimeError(f"fused forward differs from the oracle on rows {bad}")
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.__enter__()
    elapsed = loop.time_replays(args.steps, stream)
    if sampler:
        sampler.__exit__(None, None, None)
    elapsed = _max_over_ranks(elapsed, dev, world)
    if world > 1:
        dist.barrier()
    per_step = elapsed / args.steps
    per_call = per_step / CALLS_PER_STEP
    value = CALLS_PER_STEP * L * world / per_step
    del loop
    # the same workload in the exact arithmetic (the reference's PyTorch op order)
    loop_e = GraphLoop(lambda i: ops.bld_forward(xs[i % nbuf], alphas, S, out=ys[i % nbuf], arith="exact"),
                       CALLS_PER_STEP)
    for _ in range(args.warmup):
        loop_e.graph.replay()
    torch.cuda.synchronize()
    bad = _check_windows(xs[0], ys[0], S, contracted=False)
    if bad:
        raise RuntimeError(f"exact-arithmetic forward differs from the oracle on rows {bad}")
    if world > 1:
        dist.barrier()
    per_call_exact = _max_over_ranks(loop_e.time_replays(args.steps, stream), dev, world) / args.steps / CALLS_PER_STEP
    del loop_e

    # e2e through the public API: every step copies its input from pinned host
    # memory, runs the fused call and copies its result back to pinned host memory.
    # Consecutive steps are pipelined on two copy streams (step i+1's input copy
    # runs while step i's result is copied out: PCIe is full duplex), with double
    # buffers and events ordering every reuse.
    hx = [torch.randn(1, L, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    hy = [torch.empty_like(hx[0]).pin_memory() for _ in range(2)]
    d_in = [torch.empty(1, L, D, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    d_out = [torch.empty_like(d_in[0]) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    ev_back = [torch.cuda.Event() for _ in range(2)]
    for e in ev_back:
        e.record(s_out)

    def e2e_step(i):
        k = i % 2
        s_in.wait_stream(stream)  # the call that last read d_in[k] has been issued before
        with torch.cuda.stream(s_in):
            d_in[k].copy_(hx[k], non_blocking=True)
            ev_in[k].record(s_in)
        stream.wait_event(ev_in[k])
        stream.wait_event(ev_back[k])  # the copy-out that last read d_out[k] is done
        ops.bld_forward(d_in[k], alphas, S, out=d_out[k])
        ev_out[k].record(stream)
        s_out.wait_event(ev_out[k])
        with torch.cuda.stream(s_out):
            hy[k].copy_(d_out[k], non_blocking=True)
            ev_back[k].record(s_out)

    def e2e_time(n: int) -> float:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        for i in range(n):
            e2e_step(i)
        stream.wait_stream(s_out)
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / 1e3

    k_e2e = max(3, args.steps)
    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_t = _max_over_ranks(e2e_time(k_e2e), dev, world)
    last = (k_e2e - 1) % 2  # the pipelined copies delivered the oracle's result
    bad = _check_windows(hx[last], hy[last], S, contracted=True)
    if bad:
        raise RuntimeError(f"e2e pipeline result differs from the oracle on rows {bad}")
    e2e_value = L * world / (e2e_t / k_e2e)
    del d_in, d_out

    peak, peak_kind = _peaks()
    algo_bytes = 2 * tensor_bytes
    achieved = algo_bytes / per_call / 1e9
    traffic = _ncu_traffic(f"fused_fwd_bld_L{L}_D{D}_S{S}")

    sweep = None
    if not args.no_sweep and world == 1:
        sweep = []
        for Ls, steps_list in ((4096, (2, 4, 8)), (16384, range(1, 9)), (65536, range(1, 9))):
            nb = max(2, min(64, (4 * l2) // (Ls * D * esize) + 1))
            bx = [torch.randn(1, Ls, D, device=dev, dtype=torch.bfloat16) for _ in range(nb)]
            by = [torch.empty_like(bx[0]) for _ in range(nb)]
            # context: torch's device copy of the same bytes, timed the same way (the
            # launch and ramp cost every one-pass kernel of this size pays)
            gl = GraphLoop(lambda i, bx=bx, by=by, nb=nb: by[i % nb].copy_(bx[i % nb]), nb * max(1, 128 // nb))
            gl.time_replays(2, stream)
            t, n = gl.time(1024, stream)
            t /= n
            sweep.append({"L": Ls, "kernel": "torch_copy", "us_per_call": round(t * 1e6, 2),
                          "frac": round(2 * Ls * D * esize / t / 1e9 / peak, 3)})
            del gl
            for Ss in steps_list:
                for ar in ("contracted", "exact"):
                    if ar == "exact" and Ss not in (2, 4, 8):
                        continue
                    fn = (lambda i, bx=bx, by=by, Ss=Ss, nb=nb, ar=ar:
                          ops.bld_forward(bx[i % nb], [0.1] * Ss, Ss, out=by[i % nb], arith=ar))
                    gl = GraphLoop(fn, nb * max(1, 128 // nb))
                    gl.time_replays(2, stream)
                    t, n = gl.time(1024, stream)
                    t /= n
                    gbs = 2 * Ls * D * esize / t / 1e9
                    sweep.append({"L": Ls, "steps": Ss, "arith": ar, "us_per_call": round(t * 1e6, 2),
                                  "GB/s": round(gbs, 1), "frac": round(gbs / peak, 3), "tokens/s": round(Ls / t)})
                    del gl
            del bx, by
        torch.cuda.empty_cache()

    eager = _eager_host(dev) if (rank == 0 and not args.no_sweep) else None
    ref_gpu = _reference_gpu(dev, full=False) if (world == 1 and not args.no_reference_gpu) else None
    sharded = None if args.no_sharded else _sharded_parts(args, rank, world, dev)

    cpu = None
    if world == 1 and not args.no_cpu:
        cpu = cpu_reference_rate(L, D, S)

    if rank == 0:
        clocks = sampler.summary() if sampler else None
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": _config(args),
            "us_per_call": per_call * 1e6,
            "arith": "contracted: bf16 in, fp32 levels, c + alpha*lap as one fma per level (the op order of the "
                     "reference's Triton kernels); within one bf16 rounding of the exact oracle, bit-identical to "
                     "the contracted oracle on the checked windows",
            "exact": {"us_per_call": per_call_exact * 1e6, "tokens/s": L * world / per_call_exact,
                      "hbm_frac": 2 * tensor_bytes / per_call_exact / 1e9 / peak,
                      "arith": "the reference's PyTorch op order, bit-identical to the oracle"},
            "hbm_gbs": achieved, "hbm_frac": achieved / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_kind": f"{peak_kind} STREAM copy (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6650 GB/s",
                         "algorithmic_bytes_per_launch": algo_bytes},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": tensor_bytes,
                    "d2h_bytes_per_step": tensor_bytes, "steps": k_e2e, "tokens_per_step": L},
            "gpu_launches": args.steps * CALLS_PER_STEP,
            "oracle_check": "output windows (both ends, middle) bit-identical to the CPU oracle in the call's "
                            "arithmetic: device (both arithmetics) and e2e",
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        if eager is not None:
            line["eager_host_us"] = eager
        if ref_gpu is not None:
            line["reference_gpu"] = ref_gpu
        if sharded is not None:
            line["sharded"] = sharded
        if sweep is not None:
            line["sweep"] = sweep
        print(json.dumps(line), flush=True)



# ---------------------------------------------------------------------------
# other configurations of the stencil (selected with --workload)
# ---------------------------------------------------------------------------
def _max_over_ranks(t: float, dev, world: int) -> float:
    if world == 1:
        return t
    import torch.distributed as dist

    v = torch.tensor([t], device=dev, dtype=torch.float64)
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return float(v.item())


def _emit(rank, line):
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_varlen(args, rank, world, local_rank):
    """Packed prefill through the mixer: 64 sequences, lengths U[512, 8192], D=4096 bf16,
    steps 4, one varlen launch per call (each rank a replica)."""
    from types import SimpleNamespace

    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    gen = torch.Generator().manual_seed(0)
    lens = torch.randint(512, 8193, (64,), generator=gen)
    qsl = torch.zeros(65, dtype=torch.int32)
    qsl[1:] = torch.cumsum(lens, 0)
    T, D = int(qsl[-1]), args.D if args.D != 512 else 4096
    nb = 2
    xs = [torch.randn(T, D, device=dev, dtype=torch.bfloat16) for _ in range(nb)]
    md = SimpleNamespace(max_query_len=int(lens.max()), query_start_loc=qsl.to(dev), is_prefill=True)
    mixer = CtaPostAttnMixer(CtaConfig(steps=args.stencil_steps, alpha=0.1, trace=False))
    stream = torch.cuda.current_stream(dev)

    def step(i):
        mixer(xs[i % nb], attn_metadata=md)

    for i in range(args.warmup):
        step(i)
    k = min(args.steps, 200)
    t = _max_over_ranks(_time_launches(step, k, stream), dev, world)
    peak, _ = _peaks()
    per = t / k
    gbs = 2 * T * D * 2 / per / 1e9
    # the decoder layer's next line, residual + mixer(x): fused into the launch
    # (reads x and residual, writes the sum) against mixer then a torch add
    res = torch.randn(T, D, device=dev, dtype=torch.bfloat16)

    def fused(i):
        mixer(xs[i % nb], attn_metadata=md, residual=res)

    def two_pass(i):
        res + mixer(xs[i % nb], attn_metadata=md)

    for fn in (fused, two_pass):
        for i in range(3):
            fn(i)
    t_fused = _max_over_ranks(_time_launches(fused, k, stream), dev, world) / k
    t_two = _max_over_ranks(_time_launches(two_pass, k, stream), dev, world) / k
    # oracle check: the shortest, the longest and two other sequences, each run
    # through the oracle zero-padded to max_query_len (the reference rule)
    from oracle import diffusion_oracle as O

    y = mixer(xs[0], attn_metadata=md)
    torch.cuda.synchronize()
    bad = []
    for i in sorted({int(lens.argmin()), int(lens.argmax()), 0, 37}):
        a_, b_ = int(qsl[i]), int(qsl[i + 1])
        xp = torch.zeros(1, int(lens.max()), D, dtype=torch.bfloat16)
        xp[0, : b_ - a_] = xs[0][a_:b_].cpu()
        ref = O.steps_bld(xp, alpha=0.1, steps=args.stencil_steps, contracted=True)[0, : b_ - a_]
        if not torch.equal(ref, y[a_:b_].cpu()):
            bad.append(i)
    if bad:
        raise RuntimeError(f"varlen mixer differs from the oracle on sequences {bad}")
    _emit(rank, {"metric": METRIC, "value": T * world / per, "unit": "tokens/s", "n_gpus": world, "steps": k,
                 "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
                 "dtype": "bf16", "data": "synthetic",
                 "config": {"workload": "varlen_mixer", "nseq": 64, "tokens": T, "D": D,
                            "steps": args.stencil_steps, "rule": "reference zero-pad to max_query_len"},
                 "hbm_gbs": gbs, "hbm_frac": gbs / peak, "gpu_launches": k,
                 "oracle_check": "4 sequences bit-identical to the oracle (reference zero-pad rule, contracted "
                                 "arithmetic of the reference's Triton path)",
                 "residual_add": {"fused_ms": t_fused * 1e3, "two_pass_ms": t_two * 1e3,
                                  "fused_hbm_frac": 3 * T * D * 2 / t_fused / 1e9 / peak}})


def run_block(args, rank, world, local_rank):
    """PDE-Transformer LM (causal stencil) fwd+bwd: D=512, 8 heads, FFN 2048, 6 layers, pde_steps 4,
    bf16, B=1; the same model with pde_steps=0 is timed for the refinement's share."""
    from cta_b200.transformers import PDETransformerLM

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L = args.L
    torch.manual_seed(0)
    ids = torch.randint(0, 32000, (1, L), device=dev)
    tgt = torch.randint(0, 32000, (1, L), device=dev)
    mask = torch.ones(1, L, dtype=torch.long, device=dev)
    stream = torch.cuda.current_stream(dev)
    res = {}
    for pde in (args.stencil_steps, 0):
        net = PDETransformerLM(vocab_size=32000, embed_dim=512, num_heads=8, hidden_dim=2048, num_layers=6,
                               pde_steps=pde, max_length=L, dropout=0.0).to(dev, torch.bfloat16)

        def step(_i):
            out = net(ids, mask)
            loss = torch.nn.functional.cross_entropy(out.view(-1, out.shape[-1]).float(), tgt.view(-1))
            loss.backward()

        for i in range(max(3, min(args.warmup, 5))):
            step(i)
        k = max(3, min(args.steps, 10))
        res[pde] = _max_over_ranks(_time_launches(step, k, stream), dev, world) / k
        del net
        torch.cuda.empty_cache()
    per = res[args.stencil_steps]
    _emit(rank, {"metric": METRIC, "value": L * world / per, "unit": "tokens/s", "n_gpus": world, "steps": 10,
                 "warmup": 3, "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
                 "dtype": "bf16", "data": "synthetic",
                 "config": {"workload": "pde_transformer_lm_fwd_bwd", "B": 1, "L": L, "D": 512, "layers": 6,
                            "heads": 8, "ffn": 2048, "pde_steps": args.stencil_steps, "causal": True},
                 "ms_without_pde": res[0] * 1e3, "pde_share": (per - res[0]) / per})


def run_sharded(args, rank, world, local_rank):
    """Long-context stencil: bf16 x[1, L, 4096] split evenly over the ranks, steps 8,
    forward + adjoint, steps-row halos exchanged with NCCL send/recv per call."""
    from cta_b200.sharded import even_shards, sharded_diffusion

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L, D, S = args.L if args.L != 65536 else 1 << 20, 4096, args.stencil_steps if args.stencil_steps != 4 else 8
    spec = even_shards(L, world, rank)
    torch.manual_seed(1000 + rank)
    x = torch.randn(1, spec.local_len, D, device=dev, dtype=torch.bfloat16)
    g = torch.randn_like(x)
    comm = torch.cuda.Stream(device=dev, priority=-1)
    overlap = args.shard_exchange == "overlap"
    stream = torch.cuda.current_stream(dev)

    def step(_i):
        sharded_diffusion(x, spec, alpha=0.1, steps=S, comm_stream=comm, overlap=overlap)
        sharded_diffusion(g, spec, alpha=0.1, steps=S, backward=True, comm_stream=comm, overlap=overlap)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    k = max(3, min(args.steps, 20))
    t = _max_over_ranks(_time_launches(step, k, stream), dev, world)
    per = t / k
    peak, _ = _peaks()
    bytes_rank = 4 * spec.local_len * D * 2  # fwd read+write, adjoint read+write
    _emit(rank, {"metric": METRIC, "value": L / per, "unit": "tokens/s", "n_gpus": world, "steps": k,
                 "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "strong",
                 "dtype": "bf16", "data": "synthetic",
                 "config": {"workload": "sharded_fwd_bwd", "B": 1, "L": L, "D": D, "steps": S,
                            "parallelism": f"L-sharded x{world}", "halo_rows": S},
                 "hbm_gbs_per_gpu": bytes_rank / per / 1e9, "hbm_frac": bytes_rank / per / 1e9 / peak})



def run_kernels(args, rank, world, local_rank):
    """Per-kernel table on bf16 x[1, L, D] (and its [1, D, L] transpose): fused forward,
    adjoint, adjoint with d(alpha), and the [B, D, L] kernels, steps 2/4/8, graph-timed,
    inputs and outputs rotating through buffers larger than L2 (an output allocated
    inside the graph would be the same L2-resident buffer on every replay)."""
    from cta_b200 import ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L, D = args.L, args.D
    if args.mode == "kernel":
        # bare launches of ONE kernel (--kernel) for profilers: two buffers per tensor
        S = args.stencil_steps
        xs = [torch.randn(1, L, D, device=dev, dtype=torch.bfloat16) for _ in range(2)]
        gs = [torch.randn_like(xs[0]) for _ in range(2)]
        ys = [torch.empty_like(xs[0]) for _ in range(2)]
        xt = [t.transpose(1, 2).contiguous() for t in xs]
        yt = [torch.empty_like(xt[0]) for _ in range(2)]
        calls = {
            "bld_forward": lambda i: ops.bld_forward(xs[i % 2], [0.1] * S, S, out=ys[i % 2]),
            "bld_adjoint": lambda i: ops.bld_backward(gs[i % 2], [0.1] * S, S, out=ys[i % 2]),
            "bld_adjoint_dalpha": lambda i: ops.bld_backward(gs[i % 2], [0.1] * S, S, x=xs[i % 2],
                                                             need_dalpha=True, out=ys[i % 2]),
            "bdl_forward": lambda i: ops.bdl_simple(xt[i % 2], 0.1, S, out=yt[i % 2]),
            "bdl_adjoint": lambda i: ops.bdl_simple(xt[i % 2], 0.1, S, backward=True, out=yt[i % 2]),
            "bld_forward_pool": lambda i: ops.bld_forward_pool(xs[i % 2], [0.1] * S, S, pmask),
        }
        pmask = torch.ones(1, L, dtype=torch.long, device=dev)
        pmask[:, L - L // 8 :] = 0
        fn = calls[args.kernel]
        for i in range(args.warmup):
            fn(i)
        t = _time_launches(fn, args.steps, torch.cuda.current_stream(dev))
        _emit(rank, {"mode": "kernel", "kernel": args.kernel, "steps": S, "launches": args.steps,
                     "us_per_call": t / args.steps * 1e6, "L": L, "D": D})
        return
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    nb = max(2, min(16, (4 * l2) // (L * D * 2) + 1))
    xs = [torch.randn(1, L, D, device=dev, dtype=torch.bfloat16) for _ in range(nb)]
    gs = [torch.randn(1, L, D, device=dev, dtype=torch.bfloat16) for _ in range(nb)]
    ys = [torch.empty_like(xs[0]) for _ in range(nb)]
    xt = [t.transpose(1, 2).contiguous() for t in xs]
    yt = [torch.empty_like(xt[0]) for _ in range(nb)]
    stream = torch.cuda.current_stream(dev)
    peak, _ = _peaks()
    unit = L * D * 2
    rows = []

    def timed(name, steps, fn, streams):
        gl = GraphLoop(fn, nb * max(1, 32 // nb))
        t, n = gl.time(max(200, args.steps // 20), stream)
        per = t / n
        gbs = streams * unit / per / 1e9
        rows.append({"kernel": name, "steps": steps, "us": round(per * 1e6, 2), "GB/s": round(gbs, 1),
                     "frac": round(gbs / peak, 3), "bytes_per_launch": streams * unit})

    for S in range(1, 9):
        timed("bld_forward", S, lambda i, S=S: ops.bld_forward(xs[i % nb], [0.1] * S, S, out=ys[i % nb]), 2)
        timed("bld_adjoint", S, lambda i, S=S: ops.bld_backward(gs[i % nb], [0.1] * S, S, out=ys[i % nb]), 2)
        timed("bld_adjoint_dalpha", S,
              lambda i, S=S: ops.bld_backward(gs[i % nb], [0.1] * S, S, x=xs[i % nb], need_dalpha=True,
                                              out=ys[i % nb]), 3)
        if S in (2, 4, 8):
            timed("bld_forward_causal", S,
                  lambda i, S=S: ops.bld_forward(xs[i % nb], [0.1] * S, S, causal=True, out=ys[i % nb]), 2)
            timed("bdl_forward", S, lambda i, S=S: ops.bdl_simple(xt[i % nb], 0.1, S, out=yt[i % nb]), 2)
            timed("bdl_adjoint", S,
                  lambda i, S=S: ops.bdl_simple(xt[i % nb], 0.1, S, backward=True, out=yt[i % nb]), 2)
    from cta_b200 import _lib as lib_

    coef = torch.tensor([0.1], device=dev)
    for name, kind in (("pde_advection", lib_.PDE_ADVECTION), ("pde_reaction", lib_.PDE_REACTION)):
        timed(name + "_forward", 1, lambda i, kind=kind: ops.pde_step(xs[i % nb], kind, coef, coef, out=ys[i % nb]), 2)
        timed(name + "_backward", 1,
              lambda i, kind=kind: ops.pde_step(xs[i % nb], kind, coef, coef, grad_out=gs[i % nb], out=ys[i % nb]), 3)
    # the classifier's last refinement + masked mean pool: fused (x read once,
    # nothing written but [B, D]) against the stack followed by torch's pooling
    pmask = torch.ones(1, L, dtype=torch.long, device=dev)
    pmask[:, L - L // 8 :] = 0

    def stack_then_pool(i):
        y = ops.bld_forward(xs[i % nb], [0.1] * 4, 4, mask=pmask, out=ys[i % nb])
        torch.sum(y * pmask.unsqueeze(-1), dim=1) / torch.clamp(pmask.sum(dim=1, keepdim=True), min=1)

    timed("bld_forward_masked", 4, lambda i: ops.bld_forward(xs[i % nb], [0.1] * 4, 4, mask=pmask, out=ys[i % nb]), 2)
    timed("bld_forward_pool", 4, lambda i: ops.bld_forward_pool(xs[i % nb], [0.1] * 4, 4, pmask), 1)
    timed("bld_forward_then_torch_pool", 4, stack_then_pool, 1)
    _emit(rank, {"workload": "kernels", "L": L, "D": D, "dtype": "bf16", "peak_GB/s": peak, "timing":
                 "CUDA events over CUDA-graph replays, inputs rotating over >= 4x L2", "rows": rows})


def run_reference_gpu(args, rank, world, local_rank):
    """The reference's GPU path (its Triton kernels and mixer, unmodified) and
    ours on the same inputs: the full table of `_reference_gpu`, on rank 0."""
    if rank != 0:
        return
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    res = _reference_gpu(dev, full=True)
    _emit(rank, {"workload": "reference_gpu", "n_gpus": 1, **res})


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--L", type=int, default=65536)
    ap.add_argument("--D", type=int, default=512)
    ap.add_argument("--stencil-steps", type=int, default=4)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-sharded", action="store_true", help="skip the L-sharded C5 object of the default line")
    ap.add_argument("--shard-exchange", choices=["overlap", "first"], default="overlap",
                    help="sharded object: halo exchange beside the interior kernel on high-priority streams "
                         "(overlap) or before it on the compute stream (first)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip the reference's Triton GPU path timed beside ours (default line, N=1)")
    ap.add_argument("--workload", choices=["fused_fwd", "varlen", "block", "sharded", "kernels", "reference_gpu"],
                    default="fused_fwd",
                    help="fused_fwd: headline single-GPU forward; varlen: 64-sequence packed mixer, D=4096; "
                         "block: PDE-Transformer LM fwd+bwd; sharded: L=1M x 4096 split over the ranks; "
                         "kernels: per-kernel timing table; reference_gpu: the reference's Triton path "
                         "timed beside ours (rank 0)")
    ap.add_argument("--kernel", default="bld_forward",
                    choices=["bld_forward", "bld_adjoint", "bld_adjoint_dalpha", "bdl_forward", "bdl_adjoint",
                             "bld_forward_pool"],
                    help="with --workload kernels --mode kernel: the one kernel to launch")
    ap.add_argument("--mode", choices=["full", "kernel"], default="full",
                    help="kernel: only warmup + timed launches of the fused kernel (for ncu)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        # NCCL on high-priority streams: the halo exchange of the sharded path is
        # scheduled ahead of the interior kernel's pending CTAs
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank), pg_options=opts)
    try:
        {"fused_fwd": run_ours, "varlen": run_varlen, "block": run_block, "sharded": run_sharded,
         "kernels": run_kernels, "reference_gpu": run_reference_gpu}[args.workload](
            args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
