"""Benchmark: small-preset bf16 prefill (batch 8 x L=2048) through the B200 kernels.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one ``NeuraTensorModel`` forward (12 FusedSpikeBlocks, 2 sliding-
window attention layers, tied lm_head) over a [8, 2048] batch of uniform
random token ids, with the per-layer spike metrics read back.  Weights are
random-init from a seed.  With N GPUs (torchrun) the same 8 sequences are
split across the ranks (sequences are independent: strong scaling, no
collective on the data path); NCCL only gathers the per-rank spike counts.

Printed JSON (rank 0): ``value`` = tokens/s over all ranks with inputs
already in HBM, timed with CUDA events per step (max over ranks), L2 flushed
between timed steps; ``e2e`` = the same through ``InferenceEngine.run`` with
the ids copied from pinned host memory and the metrics read back each step;
``roofline`` = the selective-scan kernel on one layer of this workload;
``cpu_baseline`` = the same reference CPU path on a bounded sample.

``--impl reference`` times the reference's own PyTorch path on the host
cores (NeuraTensor 4.0.4 installed at ``baseline/_ref``; the oracle port of
that path when it is not installed), rank 0 only, one sequence per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import threading
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PRESET = "small"
GLOBAL_BATCH = 8          # sequences in the whole job, split across the ranks
SEQ = 2048
SEED = 1234


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """SM clock and clock-event reasons sampled every 10 ms while the timed region runs.

    Read-only NVML queries (the device is matched to the CUDA device by PCI
    address); nvidia-smi at its fastest interval when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, device_index: int):
        self.dev = device_index
        self.rows = []          # (sm_mhz, max_mhz, reason names)
        self.error = None
        self._stop = threading.Event()
        self._thread = None
        self._proc = None
        self._nv = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(self.dev)
        bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        try:
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.dev)

    def _sample(self):
        nv, h, mx, bits = self._nv
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        self.rows.append((float(sm), float(mx), [n for n, bit in bits if r & bit]))

    def _run_nvml(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception as e:          # keep what was sampled; say why sampling stopped
                self.error = f"nvml: {e}"
                return
            self._stop.wait(0.01)

    def __enter__(self):
        try:
            nv, h = self._nvml_handle()
            bits = [(name, getattr(nv, const)) for name, const in self.REASONS]
            self._nv = (nv, h, nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM), bits)
            self._sample()                  # at least one reading at the start of the region
            self._thread = threading.Thread(target=self._run_nvml, daemon=True)
            self._thread.start()
        except Exception as e:
            self.error = f"nvml: {e}"
            self._nv = None
            fields = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                      "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                      "clocks_event_reasons.sw_power_cap")
            try:
                self._proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={fields}",
                                               "--format=csv,noheader,nounits", "-lms", "50"],
                                              stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except Exception:
                self._proc = None
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            try:
                self._sample()              # and one at its end
            except Exception as e:
                self.error = f"nvml: {e}"
        if self._proc is not None:
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=5)
            except Exception:
                self._proc.kill()
                out = ""
            names = [n for n, _ in self.REASONS]
            for line in out.strip().splitlines():
                f = [x.strip() for x in line.split(",")]
                try:
                    self.rows.append((float(f[0]), float(f[1]),
                                      [names[i] for i in range(4) if "Active" in f[2 + i] and "Not" not in f[2 + i]]))
                except (ValueError, IndexError):
                    pass

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "error": self.error}
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": sorted({n for r in self.rows for n in r[2]}), "samples": len(self.rows)}


def _reference_package():
    """The reference package installed at baseline/_ref (NeuraTensor 4.0.4), or None."""
    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "neuratensor")):
        return None
    os.environ.setdefault("NEURATENSOR_TELEMETRY", "0")
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        import neuratensor
        from neuratensor.inference.engine import InferenceEngine  # noqa: F401
        return neuratensor
    except Exception:
        return None


# the reference's own CPU path is timed on one sequence of half the workload's length per step
REF_T_SAMPLE = 1024


class _RefCPU:
    """The reference's PyTorch path on the host cores (InferenceEngine(device="cpu",
    dtype=bf16).run, as engine.py:145-178 runs it), with its own seeded weights;
    the oracle port of that path when the reference package is not installed."""

    def __init__(self):
        import torch
        torch.set_num_threads(os.cpu_count() or 1)
        self.ref = _reference_package()
        torch.manual_seed(SEED)
        if self.ref is not None:
            from neuratensor.core.model import NeuraTensorModel as RefModel
            from neuratensor.config.presets import get_preset as ref_preset
            from neuratensor.inference.engine import InferenceEngine as RefEngine
            self.engine = RefEngine(RefModel(ref_preset(PRESET)), device="cpu", dtype=torch.bfloat16)
            self.vocab = self.engine.model.config.vocab_size
            self.kind = "reference"
        else:
            from neuratensor_b200 import NeuraTensorModel, get_preset
            from oracle import neuratensor_oracle as O
            m = NeuraTensorModel(get_preset(PRESET))
            self.p = {k: O.bf16(v) for k, v in O.params_from_state_dict(m.state_dict()).items()}
            c = m.config
            self.cfg = O.OracleConfig(vocab_size=c.vocab_size, d_model=c.d_model, n_layers=c.n_layers,
                                      d_state=c.d_state, max_seq_len=c.max_seq_len, attn_every=c.attn_every,
                                      attn_heads=c.attn_heads, attn_window=c.attn_window)
            self.vocab = c.vocab_size
            self.kind = "port"
        import numpy as np
        self.rng = np.random.default_rng(SEED)

    def forward(self, T_sample):
        import torch
        ids = self.rng.integers(0, self.vocab, (1, T_sample))
        if self.kind == "reference":
            self.engine.run(torch.from_numpy(ids), reset_state=True)
        else:
            from oracle import neuratensor_oracle as O
            O.model_forward(ids, self.p, self.cfg, None, "bf16")

    def describe(self, T_sample):
        if self.kind == "reference":
            return (f"the reference's own PyTorch path (NeuraTensor 4.0.4 from baseline/_ref, "
                    f"InferenceEngine(device='cpu', dtype=bf16).run), small preset, B=1 x T={T_sample} per step")
        return f"oracle port of the reference PyTorch path (numpy, bf16 rounding), B=1 x T={T_sample} per step"


def cpu_baseline(budget_s: float = 20.0):
    """The reference's CPU path on a bounded sample of the workload (one sequence)."""
    r = _RefCPU()
    T_sample = REF_T_SAMPLE if r.kind == "reference" else 128
    toks, t0 = 0, time.perf_counter()
    while True:
        r.forward(T_sample)
        toks += T_sample
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": toks / dt, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": r.kind,
            "sample": f"{r.describe(T_sample)}; {toks // T_sample} forwards in {dt:.1f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    r = _RefCPU()
    T_sample = REF_T_SAMPLE if r.kind == "reference" else 64
    for _ in range(args.warmup):
        r.forward(T_sample)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        r.forward(T_sample)
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    v = T_sample * args.steps / tot
    cores = os.cpu_count() or 1
    line = {"metric": "tokens/s", "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * tot / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"small preset bf16 prefill (sampled on host cores: B=1 x T={T_sample} per step)",
                       "preset": PRESET, "seq_len_sample": T_sample},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": r.kind,
                             "sample": r.describe(T_sample)},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one ssm_scan_kernel launch of
# this workload, from one ncu capture of `python bench.py --steps 1 --warmup 1 --no-cpu-baseline`
# (129,039,616 read + 25,899,776 written; the o rows are partly still in L2 when the kernel ends).
SCAN_TRAFFIC_BYTES = 154_939_392
# the same for the standalone fused LIF -> scan op (`--workload fused-op`): 640,896,768 + 438,826,752
FUSED_TRAFFIC_BYTES = 1_079_723_520


def scan_roofline(model, ids, dev, peak_gbs, peak_kind, reps=20):
    """Time the selective-scan kernel on one layer of this workload with CUDA events."""
    import torch
    from neuratensor_b200 import native
    blk = model.blocks[0]
    w, _ = blk._native_weights(torch.bfloat16, dev)
    with torch.no_grad():
        x = model.embedding(ids)
        h, gate = native.rmsnorm_in_proj(x, w["norm_w"], w["W_in"])
        spk, _ = native.lif_scan(h, w["beta"], w["threshold"])
        Wp = w["W_proj"]
        di = h.shape[-1]
        N = w["log_A"].shape[-1]
        proj = torch.nn.functional.linear(spk, Wp)
        dt = torch.nn.functional.softplus(proj[..., :di] + w["b_dt"]).contiguous()
        Bm = proj[..., di:di + N].contiguous()
        Cm = proj[..., di + N:].contiguous()
        st = torch.zeros(x.shape[0], di, N, dtype=torch.bfloat16, device=dev)
        stream = torch.cuda.current_stream(dev)
        for _ in range(3):
            native.selective_scan(spk, dt, Bm, Cm, w["log_A"], w["D"], st, gate=gate)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        ms = 0.0
        for a, b in ev:
            flush.zero_()
            a.record(stream)
            native.selective_scan(spk, dt, Bm, Cm, w["log_A"], w["D"], st, gate=gate)
            b.record(stream)
        torch.cuda.synchronize(dev)
        ms = sum(a.elapsed_time(b) for a, b in ev) / reps
    B, T = ids.shape
    M = B * T
    es = 2
    algo = M * di * es * 4 + M * 2 * N * es + 2 * B * di * N * es   # u, dt, gate, o + B|C + state in/out
    achieved = algo / (ms * 1e-3) / 1e9
    return {"kernel": "scan_kernel (selective scan + gate, one layer)", "bound": "hbm", "achieved": achieved,
            "peak": peak_gbs, "unit": "GB/s", "frac": achieved / peak_gbs, "traffic": SCAN_TRAFFIC_BYTES,
            "traffic_source": "ncu dram bytes of one launch", "algorithmic_bytes": algo, "ms_per_launch": ms,
            "peak_source": peak_kind}


def run_ours(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    from neuratensor_b200 import InferenceEngine, NeuraTensorModel, get_preset
    from neuratensor_b200 import native
    from neuratensor_b200.inference import ranks
    native.load()
    torch.manual_seed(SEED)
    model = NeuraTensorModel(get_preset(PRESET))
    eng = InferenceEngine(model, device=f"cuda:{local}", dtype=torch.bfloat16)
    model = eng.model
    # the same global batch at every world size; this rank runs rows [start, stop)
    start, stop = ranks.batch_shard(GLOBAL_BATCH, world, rank)
    if stop <= start:
        raise SystemExit(f"{world} ranks for {GLOBAL_BATCH} sequences: rank {rank} would get none")
    g = torch.Generator().manual_seed(SEED)
    host_ids = [torch.randint(0, model.config.vocab_size, (GLOBAL_BATCH, SEQ), generator=g)[start:stop]
                .contiguous().pin_memory() for _ in range(2)]
    dev_ids = [h.to(dev) for h in host_ids]
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step(i):
        logits, _, counts = model.forward_device(dev_ids[i % 2])
        return counts

    with torch.no_grad():
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        counts = None
        launches0 = native.launch_count()
        with Clocks(local) as clk:
            torch.cuda.synchronize(dev)
            for i, (a, b) in enumerate(evs):
                flush.zero_()
                a.record(stream)
                counts = step(i)
                b.record(stream)
            torch.cuda.synchronize(dev)
        launches = native.launch_count() - launches0
        if world > 1:
            dist.barrier()
        ms = sum(a.elapsed_time(b) for a, b in evs)
        clocks = clk.summary()

        # spike metrics: NCCL gather of per-rank per-layer counts (off the timed path)
        di = model.config.d_model * model.config.expand
        tot, numel = ranks.global_counts(counts, (stop - start) * SEQ * di)
        ms = ranks.max_over_ranks(ms, dev)
        metrics = model.metrics_from_counts(tot.tolist(), numel, torch.bfloat16)

        # end to end through the public API: pinned host ids -> run() -> metrics on the host
        e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps)]
        for i in range(2):
            eng.run(host_ids[i % 2], reset_state=True)
        if world > 1:
            dist.barrier()
        for i, (a, b) in enumerate(e2e_ev):
            flush.zero_()
            a.record(stream)
            r = eng.run(host_ids[i % 2], reset_state=True)
            b.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = sum(a.elapsed_time(b) for a, b in e2e_ev)
        e2e_ms = ranks.max_over_ranks(e2e_ms, dev)

        roof = None
        if rank == 0:
            peak, kind = _peaks()
            roof = scan_roofline(model, dev_ids[0], dev, peak, kind)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens = GLOBAL_BATCH * SEQ * args.steps
    value = tokens / (ms / 1000.0)
    e2e_value = tokens / (e2e_ms / 1000.0)
    cpu = None if args.no_cpu_baseline or world > 1 else cpu_baseline()
    line = {
        "metric": "tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform random ids, random-init weights, seeded)",
        "config": {"workload": f"small preset bf16 prefill, batch {GLOBAL_BATCH} x L={SEQ} split across the GPUs",
                   "preset": PRESET, "global_batch": GLOBAL_BATCH, "per_gpu_batch": stop - start, "seq_len": SEQ,
                   "parallelism": f"dp{world} (batch shards)",
                   "l2": "flushed (256 MiB write) before every timed step"},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": GLOBAL_BATCH * SEQ * 8,
                "d2h_bytes_per_step": 8 * model.config.n_layers * world,
                "metrics": "global over all ranks (InferenceEngine.run gathers the spike counts each step)"
                if world > 1 else "single process"},
        "gpu_launches": launches,
        "roofline": roof, "cpu_baseline": cpu, "clocks": clocks,
        "spike_rate": metrics["spike_rate"],
    }
    print(json.dumps(line), flush=True)


def _time_device(fn, steps, warmup, dev):
    """Average device time (ms) of fn over `steps` calls, L2 flushed before each."""
    import torch
    for _ in range(warmup):
        fn()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize(dev)
    for a, b in evs:
        flush.zero_()
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize(dev)
    return sum(a.elapsed_time(b) for a, b in evs) / steps


def run_standalone(args):
    """Standalone ops of the path on one GPU (no torchrun):
    fused-op:   LIF -> selective scan, B=16 x L=4096, d_inner 2304, d_state 64 (bf16 in, fp32 state)
    sparse-out: spike-sparse out_proj, 32768 rows x K=4096 -> 2048, row activity 10/25/50%"""
    import torch
    from neuratensor_b200 import native
    native.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(SEED)
    bf = torch.bfloat16
    peak, kind = _peaks()
    lines = []
    if args.workload == "fused-op":
        B, L, D, N = 16, 4096, 2304, 64
        x = torch.randn(B, L, D, generator=g, device=dev).to(bf)
        delta = torch.nn.functional.softplus(torch.randn(B, L, D, generator=g, device=dev) - 2.0).to(bf)
        Bm = (torch.randn(B, L, N, generator=g, device=dev) / N ** 0.5).to(bf)
        Cm = (torch.randn(B, L, N, generator=g, device=dev) / N ** 0.5).to(bf)
        log_A = torch.log(torch.arange(1, N + 1, device=dev, dtype=torch.float32)).expand(D, N).contiguous()
        Dsk = torch.ones(D, device=dev)
        beta = torch.rand(D, generator=g, device=dev) * 0.19 + 0.80
        th = torch.ones(D, device=dev)
        mem0 = torch.randn(B, D, generator=g, device=dev) * 0.5
        st0 = torch.randn(B, D, N, generator=g, device=dev) * 0.1
        cnt = torch.zeros((), dtype=torch.int64, device=dev)
        fn = lambda: native.lif_ssm_fused(x, delta, Bm, Cm, log_A, Dsk, beta, th, mem0, st0, spike_count=cnt)
        ms = _time_device(fn, args.steps, args.warmup, dev)
        algo = 1092911104
        gbs = algo / (ms * 1e-3) / 1e9
        lines.append({"metric": "tokens/s", "value": B * L / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                      "dtype": "bf16 in / fp32 state", "data": "synthetic (seeded)",
                      "config": {"workload": "fused LIF+selective scan, B=16 L=4096 d=2304 N=64"},
                      "roofline": {"kernel": "ssm_scan_kernel (LIF fused)", "bound": "hbm", "achieved": gbs,
                                   "peak": peak, "unit": "GB/s", "frac": gbs / peak, "traffic": FUSED_TRAFFIC_BYTES,
                                   "algorithmic_bytes": algo, "peak_source": kind},
                      "state_updates_per_s": B * L * D * N / (ms * 1e-3)})
    else:
        M, K, Nout = 32768, 4096, 2048
        o = torch.randn(M, K, generator=g, device=dev).to(bf)
        W = (torch.randn(Nout, K, generator=g, device=dev) * 0.02).to(bf)
        for p in (0.10, 0.25, 0.50):
            act = torch.rand(M, generator=g, device=dev) < p
            spk = ((torch.rand(M, K, generator=g, device=dev) < 0.2) & act[:, None]).to(bf)
            n_act = int(spk.any(-1).sum().item())
            fn = lambda: native.sparse_out_proj(o, spk, W)
            ms = _time_device(fn, args.steps, args.warmup, dev)
            dense = 2 * n_act > M
            rows = M if dense else n_act
            flops = 2.0 * rows * K * Nout
            byts = M * K * 2 + rows * K * 2 + K * Nout * 2 + M * Nout * 2
            lines.append({"metric": "rows/s", "value": M / (ms * 1e-3), "unit": "rows/s", "n_gpus": 1,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                          "dtype": "bf16", "data": "synthetic (seeded)",
                          "config": {"workload": f"sparse out_proj M={M} K={K} N={Nout} p={p}", "n_active": n_act,
                                     "branch": "dense" if dense else "sparse"},
                          "tflops": flops / (ms * 1e-3) / 1e12, "gbs": byts / (ms * 1e-3) / 1e9,
                          "algorithmic_bytes": byts, "flops": flops})
    for ln in lines:
        print(json.dumps(ln), flush=True)


STREAM_PRESET = "large"
STREAMS = 64              # concurrent streams in the whole job, split across the ranks
STREAM_PREFILL = 8192
STREAM_DECODE = 512


def stream_cpu_baseline(model_cfg, budget_s: float = 20.0):
    """CPU oracle port of large-preset streaming on a bounded sample: one stream,
    a 16-token prefill then greedy single-token steps with carried state."""
    import numpy as np
    import torch
    from neuratensor_b200 import NeuraTensorModel
    from oracle import neuratensor_oracle as O
    torch.manual_seed(SEED)
    m = NeuraTensorModel(model_cfg)
    p = O.params_from_state_dict(m.state_dict())
    del m
    for k in p:
        p[k] = O.bf16(p[k])
    c = model_cfg
    cfg = O.OracleConfig(vocab_size=c.vocab_size, d_model=c.d_model, n_layers=c.n_layers, d_state=c.d_state,
                         max_seq_len=c.max_seq_len, attn_every=c.attn_every, attn_heads=c.attn_heads,
                         attn_window=c.attn_window)
    rng = np.random.default_rng(SEED)
    ids = rng.integers(0, c.vocab_size, (1, 16))
    t0 = time.perf_counter()
    logits, st, _ = O.model_forward(ids, p, cfg, None, "bf16", logits_rows=np.array([15]))
    toks, steps = 16, 0
    while time.perf_counter() - t0 < budget_s:
        tok = np.argmax(logits[:, -1], axis=-1)[:, None]
        logits, st, _ = O.model_forward(tok, p, cfg, st, "bf16")
        toks += 1
        steps += 1
    dt = time.perf_counter() - t0
    return {"value": toks / dt, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"oracle (numpy, bf16-rounding emulation) {STREAM_PRESET} preset, 1 stream: 16-token "
                      f"prefill + {steps} greedy decode steps in {dt:.1f} s"}


def run_streaming(args):
    """Large-preset streaming generation: every stream prefills STREAM_PREFILL
    uniform random ids, then takes STREAM_DECODE greedy (top_k=1) single-token
    steps with carried LIF/SSM state; the streams are split across the ranks.
    One step = the whole generation for this rank's streams through
    ``NeuraTensorModel.generate`` (prefill, then the captured decode step)."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=600))
    from neuratensor_b200 import NeuraTensorModel, get_preset, native
    from neuratensor_b200.inference import ranks
    native.load()
    streams, prefill, decode = args.streams or STREAMS, args.prefill or STREAM_PREFILL, args.decode or STREAM_DECODE
    torch.manual_seed(SEED)
    cfg = get_preset(STREAM_PRESET)
    model = NeuraTensorModel(cfg).to(dev).to(torch.bfloat16).eval()
    start, stop = ranks.batch_shard(streams, world, rank)
    if stop <= start:
        raise SystemExit(f"{world} ranks for {streams} streams: rank {rank} would get none")
    g = torch.Generator().manual_seed(SEED)
    host_ids = torch.randint(0, cfg.vocab_size, (streams, prefill), generator=g)[start:stop].contiguous().pin_memory()
    stream = torch.cuda.current_stream(dev)

    def step():
        ids = host_ids.to(dev, non_blocking=True)
        torch.manual_seed(SEED)
        out, _ = model.generate(ids, max_new_tokens=decode, top_k=1)
        return out[:, prefill:].to("cpu", non_blocking=True)

    with torch.no_grad():
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        launches0 = native.launch_count()
        with Clocks(local) as clk:
            torch.cuda.synchronize(dev)
            for a, b in evs:
                a.record(stream)
                toks = step()
                b.record(stream)
            torch.cuda.synchronize(dev)
        launches = native.launch_count() - launches0
        ms = ranks.max_over_ranks(sum(a.elapsed_time(b) for a, b in evs), dev)
        # prefill alone, for the split of the step time
        pre = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(2)]
        ids = host_ids.to(dev)
        for a, b in pre:
            a.record(stream)
            model.forward_device(ids, last_only=True)
            b.record(stream)
        torch.cuda.synchronize(dev)
        pre_ms = ranks.max_over_ranks(sum(a.elapsed_time(b) for a, b in pre) / len(pre), dev)
        clocks = clk.summary()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    per_step = ms / args.steps
    tokens = streams * (prefill + decode)
    cpu = None if args.no_cpu_baseline or world > 1 else stream_cpu_baseline(cfg)
    line = {
        "metric": "tokens/s", "value": tokens / (per_step / 1000.0), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform random ids, random-init weights, seeded)",
        "config": {"workload": f"{STREAM_PRESET} preset streaming generation: {streams} streams x "
                               f"({prefill}-token prefill + {decode} greedy decode steps) split across the GPUs",
                   "preset": STREAM_PRESET, "streams": streams, "per_gpu_streams": stop - start,
                   "prefill": prefill, "decode_steps": decode, "parallelism": f"dp{world} (stream shards)",
                   "l2": "inputs larger than L2 (weights 2.7 GB, states 1.9 GB at 64 streams)"},
        "prefill_ms": pre_ms, "decode_ms_per_token": (per_step - pre_ms) / decode,
        "decode_tokens_per_s": streams * decode / ((per_step - pre_ms) / 1000.0),
        "e2e": {"value": tokens / (per_step / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": streams * prefill * 8, "d2h_bytes_per_step": int(toks.numel()) * 8 * world,
                "note": "the timed step copies the prefill ids from pinned host memory and the generated tokens back"},
        "gpu_launches": launches, "cpu_baseline": cpu, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="model", choices=["model", "fused-op", "sparse-out", "streaming"],
                    help="model: small-preset prefill (the headline); streaming: large-preset generation; "
                         "the others time one op")
    ap.add_argument("--streams", type=int, default=0, help="streaming: streams in the job (default 64)")
    ap.add_argument("--prefill", type=int, default=0, help="streaming: prefill length (default 8192)")
    ap.add_argument("--decode", type=int, default=0, help="streaming: decode steps (default 512)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "streaming":
        run_streaming(args)
    elif args.workload != "model":
        run_standalone(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
