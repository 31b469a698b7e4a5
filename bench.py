#!/usr/bin/env python3
"""Benchmark: quantized MoE decode layer, microseconds per layer per token, on 1..8 B200s.

One step = one FP8 MoE layer (the stack's layers 0-19) followed by one FP4 MoE layer (layers
20-39), each on B fresh bf16 tokens: router (fp32 logits, top-6 of 384, sigmoid, bias, x2.5),
6 routed experts + 1 FP8 shared expert (H 5120, I 2048, SwiGLU), routing-weighted combine, and at
N > 1 the fp32 all-reduce of the tensor-parallel partials (each GPU holds I/N rows of every
expert). With equal FP8 and FP4 layer counts, the mean over the two is the 40-layer stack's mean
per-layer time. Weights are seeded synthetic N(0, 0.02), generated and resident in HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Prints one JSON line (rank 0). ``value`` is device time (CUDA events on the launching stream,
max over ranks; every step streams more weight bytes than L2 holds, so no flush is needed --
``--l2-flush`` adds one); ``e2e`` is the same metric through the public API
with the step's tokens copied from pinned host memory and its outputs read back every step: the
traced decode step (``dsmoe.DecodeTrace``) when it applies, with the eager ``MoE.forward`` figure
beside it.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "tenstorrent-wormhole-deepseek-v41-flash_b200")
for _p in (ROOT, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "FP8/FP4 MoE layer us/token + HBM GB/s vs 8 TB/s peak at 1/2/4/8 B200"
UNIT = "us/layer/token"
H, I, E, TOPK = 5120, 2048, 384, 6
ROUTE_SCALE = 2.5
NOMINAL_HBM_GBS = 8000.0
DTYPE_TC = ("tcgen05: FP8 layers e4m3 x e4m3 (kind::f8f6f4, fp32 128x128 block scales on the fp32 block "
            "accumulators), FP4 layers e2m1 x e4m3 with e8m0 32-K scales (kind::mxf8f6f4.block_scale); fp32 "
            "accumulation; tokens as e4m3 hi/lo pairs")
DTYPE_FRAG = "e4m3 x e4m3 -> f32 (FP8 weights as stored, FP4 expanded to e4m3; tokens as e4m3 hi/lo pairs)"
FALLBACK_HBM_GBS = 6650.0

# algorithmic bytes (weights + scales) per expert and per router (fp32 weight + bias)
ROUTER_BYTES = E * H * 4 + E * 4  # at the configured 384 experts; scaled to --experts below
FP8_W13 = 2 * (H * I + (I // 128) * (H // 128) * 4)
FP8_W2 = H * I + (H // 128) * (I // 128) * 4
FP4_W13 = 2 * (H * I // 2 + H * I // 32)
FP4_W2 = H * I // 2 + H * I // 32


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--experts", type=int, default=E,
                    help="routed experts kept resident per layer (default 384; smaller only for profiler runs)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", choices=["both", "fp8", "fp4"], default="both",
                    help="layer formats per step (default both; one format only for profiler runs)")
    ap.add_argument("--l2-flush", action="store_true",
                    help="write 256 MiB between steps (default: off; each step already streams more than L2)")
    ap.add_argument("--cpu-budget", type=float, default=20.0, help="seconds of CPU baseline sampling")
    ap.add_argument("--mode", choices=["decode", "prefill", "sweep", "stack", "gemm"], default="decode",
                    help="decode: the headline config (default); prefill: P tokens with Zipf routing through the "
                         "tcgen05 grouped GEMMs; sweep: decode batch 1..64 and the batched path under uniform / Zipf routing")
    ap.add_argument("--tokens", type=int, default=126, help="prefill mode: tokens per layer call")
    ap.add_argument("--stack-layers", type=int, default=40,
                    help="stack mode: layers (first half FP8, second half FP4); fewer if they do not fit in HBM")
    ap.add_argument("--emulate-tp", type=int, default=1,
                    help="stack mode on one GPU: build rank 0's 1/N slice of every expert (the per-GPU kernel of "
                         "an N-GPU run, without its all-reduce); the output is labelled as emulated")
    ap.add_argument("--allreduce", choices=["p2p", "nccl"], default="p2p",
                    help="N > 1: sum the partials inside the layer kernel over NVLink peers (default) or with NCCL")
    ap.add_argument("--decode-store", choices=["tc", "frag"], default="frag",
                    help="resident store of decode layers of 1..8 tokens: the fragment layout (mma.sync kernel, "
                         "default) or the tensor-core layout (tcgen05 kernel)")
    ap.add_argument("--no-alt-store", dest="alt_store", action="store_false",
                    help="N = 1, 1..8 tokens: skip the second decode store's timing and parity (reported as "
                         "alt_store beside the line)")
    ap.add_argument("--no-stack", dest="stack_in_bench", action="store_false",
                    help="decode mode at N >= 4: skip the 40-layer stack measurement reported beside the line")
    return ap.parse_args()


DECODE_STORE = "frag"


def decode_layouts(B):
    """Resident store of a decode benchmark layer: ``--decode-store`` for 1..8 tokens, the fragment
    layout for larger batches."""
    return (DECODE_STORE,) if B <= 8 else ("frag",)


def alt_layouts(args, B, world):
    """The other decode store, kept too at N = 1 and 1..8 tokens so the line also reports it."""
    if world != 1 or B > 8 or not args.alt_store:
        return ()
    return ("frag",) if DECODE_STORE == "tc" else ("tc",)


def layer_formats(args):
    lay = getattr(args, "layers", "both")
    return ["fp8", "fp4"] if lay == "both" else [lay]


def workload_config(args, world):
    flush_l2 = getattr(args, "l2_flush", False)
    return {"workload": "one FP8 + one FP4 MoE decode layer per step (experts resident, TP over GPUs)",
            "hidden": H, "inter": I, "experts": getattr(args, "experts", E), "topk": TOPK, "shared_experts": 1, "batch": args.batch,
            "score_func": "sigmoid", "route_scale": ROUTE_SCALE, "layers_per_step": [{"fp8": "fp8-block128", "fp4": "fp4-e2m1-e8m0"}[f] for f in layer_formats(args)],
            "parallelism": f"tp{world}",
            "allreduce": (None if world == 1 else "in-kernel NVLink peer exchange (one launch per layer)"
                          if getattr(args, "allreduce", "p2p") == "p2p" else "NCCL all-reduce of fp32 partials"),
            "l2": ("flushed between steps (256 MiB write, outside the timed events)" if flush_l2 else
                   "not flushed: every step streams more weight bytes than the 126 MB L2 (read with an L2 "
                   "evict-first policy); tokens rotate through a 256-row pool")}


# ------------------------------------------------------------------ reference arm (CPU)

def _synth_module():
    """dsmoe/synth.py loaded as a plain file: the CPU arm uses its seeded quantizers (torch only) and
    must not import the dsmoe package, whose __init__ loads the CUDA library."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("_bench_synth", os.path.join(PKG_DIR, "dsmoe", "synth.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


_CPU_LAYERS = {}


def cpu_layers_setup(seed, pool=6):
    """Router at full size; the chosen experts' weights come from a pool of ``pool`` experts per
    format (expert e -> pool[e % pool]); the arithmetic per step is the full layer's. Built once per
    seed and process."""
    if seed not in _CPU_LAYERS:
        _CPU_LAYERS[seed] = _cpu_layers_build(seed, pool)
    return _CPU_LAYERS[seed]


def _cpu_layers_build(seed, pool):
    import torch
    synth = _synth_module()
    gen = torch.Generator().manual_seed(seed)
    layers = []
    for fmt in ("fp8", "fp4"):
        rw = synth.make_router(E, H, gen)
        experts = [synth.make_expert(fmt, H, I, gen) for _ in range(pool)]
        shared = synth.make_expert("fp8", H, I, gen)
        layers.append((rw, experts, shared))
    toks = synth.make_tokens(64, H, gen)
    return layers, toks


def run_cpu(args, steps, warmup, budget_s=None):
    import torch
    from oracle import cpu_baseline as CB
    cores = CB.use_all_cores()
    layers, toks = cpu_layers_setup(args.seed)
    B = args.batch

    def step(i):
        for li, (rw, experts, shared) in enumerate(layers):
            j = (2 * i + li) % (64 - B + 1)
            CB.layer(toks[j:j + B], rw.wg, rw.bias, lambda e, ex=experts: ex[e % len(ex)], shared, TOPK, ROUTE_SCALE)

    with torch.inference_mode():
        sec, n = CB.time_steps(step, steps, warmup, min_steps=1, budget_s=budget_s)
    us = sec * 1e6 / (2 * B)
    from oracle import ref_fp4lib
    sample = (f"{n} steps of {{FP8 layer + FP4 layer}} at batch {B}, torch CPU fp32 (kernel.py fp8_gemm/fp4_gemm "
              f"math, weights re-dequantized per call), FP4 unpack via "
              f"{'the reference fp4lib.c (oracle/_ref)' if ref_fp4lib.available() else 'the torch LUT'}; "
              f"{CB.cpu_model()}")
    return {"value": round(us, 2), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
            "ms_per_step": round(sec * 1e3, 3), "steps": n}


def reference_arm(args):
    rank, _, world = int(os.environ.get("RANK", 0)), 0, int(os.environ.get("WORLD_SIZE", 1))
    if rank != 0:
        return
    cb = run_cpu(args, args.steps, args.warmup)
    line = {"metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus, "steps": cb["steps"],
            "warmup": args.warmup, "ms_per_step": cb["ms_per_step"], "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, world), "impl": "reference",
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm

class ClockSampler:
    """SM clocks and throttle reasons of this rank's GPU during the timed region.

    A background ``nvidia-smi -lms 200`` runs across the region; rows whose timestamp falls inside
    [first step, last step] are kept. Timed regions are often shorter than the 200 ms period, so
    ``mark()`` -- called right after the timed steps are queued, while the GPU runs them -- also
    takes one sample, which is inside the region by construction."""
    Q = ("index,uuid,timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid, self.proc, self.path = uuid, None, None
        self.marks, self.t0, self.t1 = [], None, None

    def _cmd(self, loop):
        c = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits"]
        if self.uuid:
            c += ["-i", self.uuid]
        return c + (["-lms", "200"] if loop else [])

    def __enter__(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(self._cmd(True), stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        self.t0 = time.time()
        return self

    def mark(self):
        """One sample now. NVML in-process (tens of microseconds, so it can be taken while queued
        steps run); nvidia-smi when NVML is unavailable. Reads only."""
        try:
            import datetime
            import pynvml as N
            N.nvmlInit()
            h = N.nvmlDeviceGetHandleByUUID(self.uuid) if self.uuid else N.nvmlDeviceGetHandleByIndex(0)
            sm = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
            smax = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            pw = N.nvmlDeviceGetPowerUsage(h) / 1000.0
            r = N.nvmlDeviceGetCurrentClocksEventReasons(h)
            act = lambda bit: "Active" if r & bit else "Not Active"
            ts = datetime.datetime.now().strftime("%Y/%m/%d %H:%M:%S.%f")
            self.marks.append(", ".join([
                "0", self.uuid or "", ts, str(sm), str(smax), f"{pw:.2f}", hex(r),
                act(N.nvmlClocksEventReasonHwSlowdown), act(N.nvmlClocksEventReasonHwThermalSlowdown),
                act(N.nvmlClocksEventReasonSwThermalSlowdown), act(N.nvmlClocksEventReasonSwPowerCap)]))
            return
        except Exception:
            pass
        try:
            out = subprocess.run(self._cmd(False), capture_output=True, text=True, timeout=10).stdout
            self.marks += [ln for ln in out.splitlines() if ln.strip()]
        except (OSError, subprocess.SubprocessError):
            pass

    def __exit__(self, *exc):
        self.t1 = time.time()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    @staticmethod
    def _parse(line):
        f = [c.strip() for c in line.split(",")]
        if len(f) < 11:
            return None
        try:
            import datetime
            ts = datetime.datetime.strptime(f[2], "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            ts = None
        return f, ts

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                r = self._parse(line)
                if r and r[1] is not None and self.t0 is not None and self.t0 <= r[1] <= (self.t1 or r[1]):
                    rows.append(r[0])
            os.unlink(self.path)
        except OSError:
            pass
        rows += [r[0] for r in map(self._parse, self.marks) if r]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        num = lambda v: float(v) if v.replace(".", "").isdigit() else None
        sm = [num(r[3]) for r in rows if num(r[3]) is not None]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[7:11]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(rows[0][4]),
                "reasons": reasons, "samples": len(rows), "in_region": "timestamped background samples inside "
                "the timed region plus one in-process NVML sample taken while the queued timed steps run"}


def _oracle_expert(ew):
    from oracle import moe as OM
    n = lambda t: t.cpu().numpy()
    return OM.QuantExpert(ew.fmt, n(ew.w1), n(ew.s1), n(ew.w3), n(ew.s3), n(ew.w2), n(ew.s2))


def check_parity(args, layers, refs, layer_launch, xin, yout, idx_st, comm, rank, world, dev):
    """Outside the timed region: one call of every layer on the first token variant, checked
    (a) at N > 1 for the same bits on every rank (all-gather), (b) on rank 0 against the oracle
    holding the experts that call routes to (max-abs-rel and cosine of the bf16 output against the
    fp32-dequant reference, router indices bit-exact); at N > 1 with the peer exchange, also the
    stand-alone row all-reduce against an fp32 NCCL sum rounded to bf16 (bit-equal, same bits on every
    rank). Every rank takes the same collective steps."""
    import numpy as np
    import torch
    import torch.distributed as dist
    out = {"tolerance": {"max_abs_rel": 1e-2, "cosine": 0.9999}}
    ok = True
    for li, nm in enumerate(layer_formats(args)):
        layer_launch(li, 0)
        torch.cuda.synchronize(dev)
        y = yout[li].clone()
        ent = {}
        if world > 1:
            allv = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(allv, y)
            ent["same_bits_all_ranks"] = all(torch.equal(allv[0], v) for v in allv)
            ok &= ent["same_bits_all_ranks"]
        if rank == 0:
            from oracle import moe as OM
            yr, ridx, _ = OM.moe_forward(refs[li], xin[li][0].float().cpu().numpy())
            mar, cos = OM.compare(y.float().cpu().numpy(), yr)
            ent.update(idx_match=bool(np.array_equal(idx_st[li][0].cpu().numpy(), ridx)), max_abs_rel=mar,
                       cosine=cos, tokens=int(y.shape[0]))
            ok &= ent["idx_match"] and mar < 1e-2 and cos > 0.9999
        out[f"{nm}_layer"] = ent
    if world > 1 and comm is not None:  # the attention-output all-reduce on the same comm
        rows_ok = True
        for Br in (1, 5, 8):
            g = torch.Generator(device=dev).manual_seed(args.seed + 100 * Br + rank)
            xr = torch.randn((Br, H), generator=g, device=dev).to(torch.bfloat16)
            yr = comm.allreduce(xr)
            comm.check()
            ref = xr.float()
            dist.all_reduce(ref)
            rows_ok &= bool(torch.equal(yr, ref.to(torch.bfloat16)))
            allv = [torch.empty_like(yr) for _ in range(world)]
            dist.all_gather(allv, yr)
            rows_ok &= all(torch.equal(allv[0], v) for v in allv)
        out["allreduce_rows"] = {"equals_fp32_nccl_sum_in_bf16": rows_ok, "rows": [1, 5, 8]}
        ok &= rows_ok
    for m in layers:
        m.check(args.batch)
    if world > 1:  # rank 0's oracle verdict on every rank
        t = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok = bool(t.item())
    out["ok"] = bool(ok)
    return out


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def ours(args):
    import torch
    import torch.distributed as dist
    import dsmoe
    from dsmoe import _lib as L
    from dsmoe.tp import env_rank_world, max_over_ranks

    rank, local, world = env_rank_world()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    B = args.batch
    if not 1 <= B <= L.MAX_DECODE_TOKENS:
        raise SystemExit(f"--batch must be in 1..{L.MAX_DECODE_TOKENS}")

    # ---- tokens first (their own generator), so that the parity step's routing is known before the
    # experts are generated and rank 0 can keep the experts it needs for the oracle check
    t_setup = time.time()
    pool = 256
    toks = dsmoe.make_tokens(pool + B, H, torch.Generator(device=dev).manual_seed(args.seed + 7), device=dev)
    n_layers = len(layer_formats(args))
    NV = 7  # token variants: step s uses variant s % NV, so routing changes from step to step
    xin = [[toks[(v * n_layers + li) * 7 % pool:][:B] for v in range(NV)] for li in range(n_layers)]
    # ---- resident layers (same seed on every rank: rank r packs its slice)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    layers, refs = [], []
    for li, fmt in enumerate(layer_formats(args)):
        NE = args.experts
        m = dsmoe.MoE(H, I, NE, TOPK, fmt, "sigmoid", ROUTE_SCALE, rank=rank, world=world, device=dev, max_tokens=B,
                      layouts=decode_layouts(B) + alt_layouts(args, B, world))
        m.use_decode_store(decode_layouts(B)[0])
        rw = dsmoe.make_router(NE, H, gen, device=dev)
        m.load_router(rw)
        sh = dsmoe.make_expert("fp8", H, I, gen, device=dev)
        m.load_shared(sh)
        need = set()
        if rank == 0:  # the experts the oracle routes the parity step's tokens to
            from oracle import moe as OM
            ridx, _, _ = OM.route(xin[li][0].float().cpu().numpy(), rw.wg.cpu().numpy(), rw.bias.cpu().numpy(), TOPK,
                                  "sigmoid", ROUTE_SCALE)
            need = set(ridx.ravel().tolist())
        kept = {}
        for e in range(NE):
            ew = dsmoe.make_expert(fmt, H, I, gen, device=dev)
            m.load_expert(e, ew)
            if e in need:
                kept[e] = ew.to("cpu")
            del ew
        if rank == 0:
            refs.append(OM.MoELayer(rw.wg.cpu().numpy(), rw.bias.cpu().numpy(),
                                    [_oracle_expert(kept[e]) if e in kept else None for e in range(NE)],
                                    _oracle_expert(sh.to("cpu")), TOPK, "sigmoid", ROUTE_SCALE))
        del rw, sh, kept
        layers.append(m)
    torch.cuda.synchronize()
    comm = None
    if world > 1 and args.allreduce == "p2p":
        from dsmoe.tp import PeerComm
        comm = PeerComm(H, device=dev)
        for m in layers:
            m.use_comm(comm)
    setup_s = time.time() - t_setup

    flush = torch.empty(256 * 1024 * 1024 if args.l2_flush else 1, dtype=torch.uint8, device=dev)
    K, W = args.steps, args.warmup
    stream = torch.cuda.current_stream(dev)
    idx_st = [[torch.zeros((B, TOPK), dtype=torch.int64, device=dev) for _ in range(NV)] for _ in range(n_layers)]
    idx_log = torch.zeros((K + W, n_layers, B, TOPK), dtype=torch.int64, device=dev)
    part = [torch.empty((B, H), dtype=torch.float32, device=dev) for _ in range(n_layers)]
    yout = [torch.empty((B, H), dtype=torch.bfloat16, device=dev) for _ in range(n_layers)]
    p2p = comm is not None and all(
        L.lib.dsmoe_moe_allreduce_supported(m._layer, comm.handle, L.ptr(xin[0][0]), B) for m in layers)
    launches_per_layer = (1 if B <= 8 else 5) + (1 if world > 1 and not p2p else 0)

    def layer_launch(li, v):
        m = layers[li]
        st_ = torch.cuda.current_stream(dev).cuda_stream
        if p2p:  # the layer kernel sums the ranks' partials itself
            L.call("dsmoe_moe_decode_allreduce", m._layer, comm.handle, L.ptr(xin[li][v]), B, None,
                   L.ptr(yout[li]), L.DTYPE_BF16, L.ptr(idx_st[li][v]), None, None, L.ptr(m.workspace),
                   m.workspace.numel(), st_)
            return
        y_t, y_dt = (part[li], L.DTYPE_F32) if world > 1 else (yout[li], L.DTYPE_BF16)
        L.call("dsmoe_moe_decode", m._layer, L.ptr(xin[li][v]), B, None, L.ptr(y_t), y_dt,
               L.ptr(idx_st[li][v]), None, None, L.ptr(m.workspace), m.workspace.numel(), st_)
        if world > 1:
            dist.all_reduce(part[li])
            L.call("dsmoe_f32_to_bf16", L.ptr(part[li]), L.ptr(yout[li]), part[li].numel(), st_)

    if world > 1:  # ranks enter the first layer together (the in-kernel exchange's waits are bounded)
        dist.barrier()
        torch.cuda.synchronize()
    # eager warm-up (first-call set-up, NCCL communicators), then one CUDA graph per token variant
    # holding the whole step (every layer) with timestamp nodes before, between and after the layers:
    # the timed steps replay graphs, so no host-side launch work sits between the kernels
    for v in range(NV):
        for li in range(n_layers):
            layer_launch(li, v)
    torch.cuda.synchronize()
    parity = check_parity(args, layers, refs, layer_launch, xin, yout, idx_st, comm, rank, world, dev)
    gev =[[torch.cuda.Event(enable_timing=True, external=True) for _ in range(n_layers + 1)] for _ in range(NV)]
    pev = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(2)] for _ in range(NV)]
    graphs, pgraphs = None, None
    timing_mode = ("cuda-graph replay: the K timed steps (every layer of each, token variants in step order) "
                   "captured as one graph and replayed once between two CUDA events (barrier + synchronize "
                   "before, synchronize after), so consecutive layer kernels overlap (programmatic dependent "
                   "launch); the per-layer split from a second pass of per-step graphs with timestamp nodes "
                   "between the layers, synchronized per step")
    try:
        graphs = [torch.cuda.CUDAGraph() for _ in range(NV)]
        pgraphs = [torch.cuda.CUDAGraph() for _ in range(NV)]
        for v in range(NV):
            with torch.cuda.graph(graphs[v]):
                for li in range(n_layers):
                    gev[v][li].record()
                    layer_launch(li, v)
                gev[v][n_layers].record()
            with torch.cuda.graph(pgraphs[v]):
                pev[v][0].record()
                for li in range(n_layers):
                    layer_launch(li, v)
                pev[v][1].record()
        torch.cuda.synchronize()
    except Exception as ex:  # pragma: no cover - depends on the driver
        graphs, pgraphs, timing_mode = None, None, f"eager launches (graph capture failed: {type(ex).__name__})"
        torch.cuda.synchronize()
    eev = [[torch.cuda.Event(enable_timing=True) for _ in range(n_layers + 1)] for _ in range(NV)]
    layer_t = [[] for _ in range(n_layers)]
    step_t = []

    def step(s, timed, split=False):
        v = s % NV
        if graphs is not None:
            if split:
                graphs[v].replay()
                e_ = gev[v]
            else:
                pgraphs[v].replay()
                e_ = pev[v]
        else:
            e_ = eev[v]
            for li in range(n_layers):
                e_[li].record(stream)
                layer_launch(li, v)
            e_[n_layers].record(stream)
        torch.cuda.synchronize()  # the variant's timestamps are re-written by its next replay
        if timed:
            if split or graphs is None:
                for li in range(n_layers):
                    layer_t[li].append(e_[li].elapsed_time(e_[li + 1]))
            if not split:
                step_t.append(e_[0].elapsed_time(e_[-1]))
        if not split:
            for li in range(n_layers):
                idx_log[s, li].copy_(idx_st[li][v])
        if args.l2_flush:
            flush.zero_()

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass

    if world > 1:
        dist.barrier()
    for s in range(W):
        step(s, False)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
        dist.barrier()  # the barrier's own work has completed on every rank before the first step
    torch.cuda.synchronize()
    # The K timed steps run back to back (no host synchronisation between them), bracketed by a
    # barrier and a synchronize: at N > 1 the ranks then run in lockstep through the in-kernel
    # exchange, and a host-side delay on one rank is not charged to every step.
    # With graphs, the K steps (their token variants in step order) are one graph, as a decode loop
    # replays one graph per token: no launch gap between steps.
    kgraph = None
    if graphs is not None:
        try:
            kgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(kgraph):
                for s in range(W, W + K):
                    for li in range(n_layers):
                        layer_launch(li, s % NV)
            torch.cuda.synchronize()
        except Exception:  # pragma: no cover - depends on the driver
            kgraph = None
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()
            dist.barrier()
        torch.cuda.synchronize()
    t_beg, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(uuid) as clk:
        t_beg.record(stream)
        if kgraph is not None:
            kgraph.replay()
        else:
            for s in range(W, W + K):
                v = s % NV
                if graphs is not None:
                    pgraphs[v].replay()
                else:
                    for li in range(n_layers):
                        layer_launch(li, v)
        t_end.record(stream)
        if rank == 0:
            clk.mark()  # while the queued steps run
        torch.cuda.synchronize()
    step_t = [t_beg.elapsed_time(t_end) / K] * K
    for s in range(W, W + K):  # every replay of a token variant routes the same way
        for li in range(n_layers):
            idx_log[s, li].copy_(idx_st[li][s % NV])
    if graphs is not None:  # second pass: the per-layer split (timestamp nodes between the layers)
        for s in range(W):
            step(s, False, split=True)
        for s in range(W, W + K):
            step(s, True, split=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for m in layers:
        m.check(B)
    graphs = pgraphs = kgraph = None  # released before the process group goes away

    # ---- per-step and per-layer device times
    step_ms = step_t
    layer_ms = {li: layer_t[li] for li in range(n_layers)}
    ms_per_step = max_over_ranks(sum(step_ms) / K, dev)
    value = ms_per_step * 1e3 / (n_layers * B)

    # unique experts per step -> algorithmic bytes
    uniq = [[len(set(idx_log[s, li].flatten().tolist())) for li in range(n_layers)] for s in range(W, W + K)]
    names = layer_formats(args)
    w13_b = {"fp8": FP8_W13, "fp4": FP4_W13}
    w2_b = {"fp8": FP8_W2, "fp4": FP4_W2}
    kern = {}
    for li, nm in enumerate(names):
        u = statistics.mean(uq[li] for uq in uniq)
        b13 = (u * w13_b[nm] + FP8_W13) / world
        b2 = (u * w2_b[nm] + FP8_W2) / world
        byts = args.experts * (H * 4 + 4) + b13 + b2  # router rows + bias, replicated on every rank
        t = statistics.mean(layer_ms[li])
        kern[f"{nm}_layer"] = {"us": round(t * 1e3, 2), "bytes": int(byts), "gbs": round(byts / (t * 1e-3) / 1e9, 1),
                               "launches": launches_per_layer}
    tot_us = sum(v["us"] for v in kern.values())
    for v in kern.values():
        v["share"] = round(v["us"] / tot_us, 3) if tot_us else None
    step_bytes = sum(v["bytes"] for v in kern.values())
    dom_name = max((k for k in kern if kern[k]["bytes"]), key=lambda k: kern[k]["us"])
    dom = kern[dom_name]
    peak, peak_kind = measured_peak()
    achieved = dom["gbs"]
    traffic = read_traffic(dom_name, B, world)

    # ---- the other decode store (N = 1): the same layers, tokens and routing through its kernel
    alt = None
    alts = alt_layouts(args, B, world)
    if alts:
        for m in layers:
            m.use_decode_store(alts[0])
        aparity = check_parity(args, layers, refs, layer_launch, xin, yout, idx_st, comm, rank, world, dev)
        ams = variant_times([lambda v, li=li: layer_launch(li, v) for li in range(n_layers)], NV, K, W, dev)
        for m in layers:
            m.check(B)
            m.use_decode_store(decode_layouts(B)[0])
        akern = {}
        for li, nm in enumerate(names):
            t = ams[li]
            byts = kern[f"{nm}_layer"]["bytes"]
            akern[f"{nm}_layer"] = {"us": round(t * 1e3, 2), "bytes": byts, "gbs": round(byts / (t * 1e-3) / 1e9, 1)}
        alt = {"store": alts[0], "dtype": DTYPE_TC if alts[0] == "tc" else DTYPE_FRAG, "kernels": akern,
               "us_per_layer_token": round(sum(ams) * 1e3 / (n_layers * B), 3), "parity": aparity,
               "timing": "CUDA graphs per token variant with timestamp nodes between the layers, replayed round-robin"}

    # ---- e2e through the public API: every step copies its layers' tokens from pinned host memory
    # (one copy for the step), runs MoE.forward per layer and reads every layer's output back
    xh = torch.empty((NV, n_layers * B, H), dtype=torch.bfloat16).pin_memory()
    for v in range(NV):
        for li in range(n_layers):
            xh[v, li * B:(li + 1) * B].copy_(xin[li][v].cpu())
    yh = [torch.empty((B, H), dtype=torch.bfloat16).pin_memory() for _ in range(n_layers)]
    xd = torch.empty((n_layers * B, H), dtype=torch.bfloat16, device=dev)

    def e2e_step(s):
        xd.copy_(xh[s % NV], non_blocking=True)
        for li, m in enumerate(layers):
            yh[li].copy_(m.forward(xd[li * B:(li + 1) * B]), non_blocking=True)
        torch.cuda.synchronize()

    def e2e_time(step_fn):
        for s in range(W):
            step_fn(s)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for s in range(K):
            step_fn(W + s)
        return max_over_ranks((time.perf_counter() - t0) * 1e3 / K, dev) * 1e3 / (n_layers * B)

    # eager: MoE.forward per layer per step
    e2e_eager = e2e_time(e2e_step)
    # traced: dsmoe.DecodeTrace (the reference's traced decode step); the step's host tokens are
    # copied into the trace's pinned input, and the graph copies them in and every output out
    # Every rank takes the same collective steps: the trace is timed only if every rank built it,
    # and its verdict is agreed before it is used (the replays and the eager check run the exchange).
    e2e_traced, trace_err = None, None
    if B <= 8 and (world == 1 or comm is not None):
        tr = None
        try:
            tr = dsmoe.DecodeTrace(layers, B)
        except Exception as ex:  # reported in the line; the eager figure stands
            trace_err = repr(ex)[:200]
        if max_over_ranks(1.0 if tr is None else 0.0, dev) == 0.0:
            xv = xh.view(NV, n_layers, B, H)
            e2e_traced = e2e_time(lambda s: tr.step(xv[s % NV]))
            bad = 0.0
            try:
                tr.check()
            except L.DsmoeError as ex:
                trace_err, bad = repr(ex)[:200], 1.0
            # the trace's last step equals the eager forward on its tokens (every layer on every rank)
            same = [torch.equal(tr.y_host[li], layers[li].forward(xv[(W + K - 1) % NV, li].to(dev)).cpu())
                    for li in range(n_layers)]
            if not all(same):
                trace_err, bad = "traced output differs from MoE.forward", 1.0
            if max_over_ranks(bad, dev) != 0.0:
                trace_err = trace_err or "the trace failed on another rank"
        elif trace_err is None:
            trace_err = "the trace could not be built on another rank"
        if tr is not None:
            tr.release()
    if trace_err is not None:
        e2e_traced = None
    e2e_val = e2e_traced if e2e_traced is not None else e2e_eager

    # ---- the 40-layer resident stack (config 4) when it fits: layers 2..39 hold copies of the two
    # benchmark layers' expert bytes in their own memory, each with its own router
    stack40 = None
    if world >= 4 and args.stack_in_bench:
        stack40 = stack_from_layers(args, layers, comm, dev, rank, world, 40)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = run_cpu(args, steps=1000, warmup=1, budget_s=args.cpu_budget)
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        by_b = {}
        for Bc in (1, 4, 8):  # BASELINE's CPU plan: the same layer pair at batch 1, 4 and 8
            a2 = argparse.Namespace(**{**vars(args), "batch": Bc})
            r = run_cpu(a2, steps=1000, warmup=1, budget_s=args.cpu_budget / 3)
            by_b[str(Bc)] = {"value": r["value"], "unit": UNIT, "ms_per_step": r["ms_per_step"], "steps": r["steps"]}
        cpu["by_batch"] = by_b

    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(ms_per_step, 5), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE_TC if decode_layouts(B) == ("tc",) else DTYPE_FRAG,
            "data": "synthetic (seeded N(0,0.02) weights quantized per the config, N(0,1) bf16 tokens)",
            "config": workload_config(args, world),
            "hbm_gbs": round(step_bytes / (ms_per_step * 1e-3) / 1e9, 1),
            "hbm_frac_of_8tbs": round(step_bytes / (ms_per_step * 1e-3) / 1e9 / NOMINAL_HBM_GBS, 3),
            "hbm_frac_of_measured": round(step_bytes / (ms_per_step * 1e-3) / 1e9 / peak, 3),
            "bytes_per_step_per_gpu": int(step_bytes),
            "unique_experts_per_layer": [round(statistics.mean(uq[li] for uq in uniq), 2) for li in range(n_layers)],
            "kernels": kern,
            "roofline": {"kernel": dom_name, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 3) if achieved else None,
                         "peak_source": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 3), "unit": UNIT, "h2d_bytes_per_step": n_layers * B * H * 2,
                    "d2h_bytes_per_step": n_layers * B * H * 2,
                    "api": "dsmoe.DecodeTrace.step" if e2e_traced is not None else "dsmoe.MoE.forward",
                    "eager_forward": round(e2e_eager, 3),
                    "traced": round(e2e_traced, 3) if e2e_traced is not None else None,
                    "trace_error": trace_err,
                    "timing": "host wall clock per step (max over ranks), tokens from pinned host memory "
                              "in and every layer's output out each step"},
            "gpu_launches": K * n_layers * launches_per_layer,
            "parity": parity,
            "alt_store": alt,
            "stack40_ms_per_token": stack40["ms_per_token"] if stack40 else None,
            "stack40": stack40,
            "timing": timing_mode,
            "clocks": clocks,
            "setup_s": round(setup_s, 1),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def read_traffic(kernel_name, B, world):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if present.

    The summary file lists lines ``traffic <kernel> b<B> tp<N> <bytes>``."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    try:
        for line in open(path):
            f = line.split()
            if len(f) == 5 and f[0] == "traffic" and f[1] == kernel_name and f[2] == f"b{B}" and f[3] == f"tp{world}":
                return int(f[4])
    except OSError:
        pass
    return None


def build_layers(args, dev, rank, world, fmts, max_tokens):
    import torch
    import dsmoe
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    layers = []
    for fmt in fmts:
        m = dsmoe.MoE(H, I, args.experts, TOPK, fmt, "sigmoid", ROUTE_SCALE, rank=rank, world=world, device=dev,
                      max_tokens=max_tokens)
        m.load_router(dsmoe.make_router(args.experts, H, gen, device=dev))
        m.load_shared(dsmoe.make_expert("fp8", H, I, gen, device=dev))
        for e in range(args.experts):
            m.load_expert(e, dsmoe.make_expert(fmt, H, I, gen, device=dev))
        layers.append(m)
    return layers, gen


def graph_times(fns, steps, warmup, dev):
    """Capture fns (one per layer) into one CUDA graph with timestamp nodes between them; replay it
    warmup + steps times (sync per replay); per-fn mean ms over the timed replays."""
    import torch
    for f in fns:
        f()
    torch.cuda.synchronize(dev)
    ev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(fns) + 1)]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i, f in enumerate(fns):
            ev[i].record()
            f()
        ev[-1].record()
    torch.cuda.synchronize(dev)
    t = [[] for _ in fns]
    for s in range(warmup + steps):
        g.replay()
        torch.cuda.synchronize(dev)
        if s >= warmup:
            for i in range(len(fns)):
                t[i].append(ev[i].elapsed_time(ev[i + 1]))
    del g
    return [statistics.mean(x) for x in t]


def variant_times(fns, NV, steps, warmup, dev):
    """Per-fn mean ms: fns[i](v) launches layer i on token variant v; one CUDA graph per variant with
    timestamp nodes between the layers, replayed round-robin over the variants (sync per replay)."""
    import torch
    for v in range(NV):
        for f in fns:
            f(v)
    torch.cuda.synchronize(dev)
    evs = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(fns) + 1)] for _ in range(NV)]
    gs = [torch.cuda.CUDAGraph() for _ in range(NV)]
    for v in range(NV):
        with torch.cuda.graph(gs[v]):
            for i, f in enumerate(fns):
                evs[v][i].record()
                f(v)
            evs[v][-1].record()
    torch.cuda.synchronize(dev)
    t = [[] for _ in fns]
    for s in range(warmup + steps):
        v = s % NV
        gs[v].replay()
        torch.cuda.synchronize(dev)
        if s >= warmup:
            for i in range(len(fns)):
                t[i].append(evs[v][i].elapsed_time(evs[v][i + 1]))
    del gs
    return [statistics.mean(x) for x in t]


def uniform_routing(P, E, k, gen, route_scale=ROUTE_SCALE):
    import torch
    idx = torch.stack([torch.randperm(E, generator=gen)[:k] for _ in range(P)]).to(torch.int64)
    w = torch.rand((P, k), generator=gen) + 0.5
    return idx, (w / w.sum(1, keepdim=True) * route_scale).to(torch.float32)


def prefill_mode(args):
    """Config: one FP8 and one FP4 layer (384 experts, full size) on P tokens with Zipf(1.1)
    routing, through the tcgen05 grouped GEMMs (the reference's prefill_batched)."""
    import torch
    import dsmoe
    from dsmoe.tp import env_rank_world
    rank, local, world = env_rank_world()
    if world != 1:
        raise SystemExit("--mode prefill runs on one GPU")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    P = args.tokens
    layers, _ = build_layers(args, dev, 0, 1, layer_formats(args), max_tokens=8)
    gen = torch.Generator().manual_seed(args.seed + 1)
    x = dsmoe.make_tokens(P, H, gen).to(dev)
    idx, wt = dsmoe.zipf_routing(P, args.experts, TOPK, gen)
    uniq = len(set(idx.flatten().tolist()))
    idx_d, wt_d = idx.to(dev), wt.to(dev)
    ms = graph_times([lambda m=m: m.prefill(x, idx_d, wt_d) for m in layers], args.steps, args.warmup, dev)
    for m in layers:
        m.prefill_check(P)
    peak, peak_kind = measured_peak()
    kern = {}
    w13_b = {"fp8": FP8_W13, "fp4": FP4_W13}
    w2_b = {"fp8": FP8_W2, "fp4": FP4_W2}
    flops = 2.0 * 3 * H * I * (P * TOPK + P)
    for nm, t in zip(layer_formats(args), ms):
        byts = uniq * (w13_b[nm] + w2_b[nm]) + FP8_W13 + FP8_W2
        kern[f"{nm}_prefill"] = {"us": round(t * 1e3, 1), "us_per_token": round(t * 1e3 / P, 3), "bytes": int(byts),
                                 "gbs": round(byts / (t * 1e-3) / 1e9, 1),
                                 "hbm_frac_of_measured": round(byts / (t * 1e-3) / 1e9 / peak, 3),
                                 "tflops": round(flops / (t * 1e-3) / 1e12, 2)}
    line = {"mode": "prefill", "metric": "prefill MoE layer us/token (tcgen05 grouped GEMMs)",
            "value": round(statistics.mean(ms) * 1e3 / P, 3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False,
            "config": {"workload": f"prefill: {P} tokens, Zipf(1.1) routing over {args.experts} experts "
                                   f"(seeded), one FP8 + one FP4 layer", "tokens": P, "pairs": P * TOPK,
                       "unique_experts": uniq, "max_tokens_per_expert": int(idx.flatten().bincount().max())},
            "kernels": kern, "peak_hbm_gbs": peak, "peak_source": peak_kind,
            "timing": "cuda-graph replay per step (timestamp nodes between layers)"}
    print(json.dumps(line), flush=True)


def gemm_mode(args):
    """The kernel-surface GEMMs (fp8_gemm / fp4_gemm, dsv41/ref/kernel.py:105-112) at a DeepSeek linear
    shape, N = K = 5120, for M in {1, 126, 2048} tokens: e4m3 activations with fp32 scales per 128-K
    block (act_quant's output, the form model.py passes), bf16 output. Enough distinct weight
    matrices rotate through the timed calls that every call reads its weights from HBM, not L2.
    Each call is one launch; the calls are replayed from a CUDA graph and timed with CUDA events.
    ``cublas_bf16_us`` is torch.matmul of bf16 activations with weights already dequantized to bf16
    (the same flops, twice the weight bytes of FP8), for context."""
    import torch
    import dsmoe  # noqa: F401  (loads libdsmoe.so)
    from dsmoe import _lib as L
    from dsmoe import synth
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N = K = H
    peak, peak_kind = measured_peak()
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
        tf_peak = float(json.load(f).get("bf16_tflops", 1590.0))
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    res = {}
    for fmt in ("fp8", "fp4"):
        w = torch.randn((N, K), generator=gen, device=dev) * 0.02
        q, sc = synth.quant_fp8_block(w) if fmt == "fp8" else synth.quant_fp4_e8m0(w)
        wbytes = q.numel() + sc.numel() * sc.element_size()
        nmat = max(2, -(-3 * 126 * 2 ** 20 // wbytes))  # > 3x L2 in rotation
        qs = [q.clone() for _ in range(nmat)]
        scs = [sc.clone() for _ in range(nmat)]
        del w
        fn = L.lib.dsmoe_fp8_gemm if fmt == "fp8" else L.lib.dsmoe_fp4_gemm
        for M in (1, 126, 2048):
            x = torch.randn((M, K), generator=gen, device=dev) * 2
            xb = x.view(M, K // 128, 128)
            a_s = (xb.abs().amax(-1).clamp(min=1e-4) / 448.0).contiguous()
            xq = (xb / a_s.unsqueeze(-1)).clamp(-448, 448).to(torch.float8_e4m3fn).view(M, K).view(torch.uint8)
            out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            st = torch.cuda.current_stream(dev).cuda_stream
            call = lambda i: L.check(fn(xq.data_ptr(), L.DTYPE_E4M3, a_s.data_ptr(), M, K, qs[i].data_ptr(),
                                        scs[i].data_ptr(), N, out.data_ptr(), L.DTYPE_BF16,
                                        torch.cuda.current_stream(dev).cuda_stream))
            call(0)  # first call outside capture (the split-K workspace is allocated here)
            torch.cuda.synchronize(dev)
            reps = nmat
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for r in range(reps):
                    call(r % nmat)
            for _ in range(max(3, args.warmup)):
                g.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                g.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            us = e0.elapsed_time(e1) * 1e3 / (args.steps * reps)
            del g
            flops = 2.0 * M * N * K
            byts = wbytes + M * K + M * (K // 128) * 4 + M * N * 2
            r = {"us": round(us, 2), "bytes": int(byts), "gbs": round(byts / (us * 1e-6) / 1e9, 1),
                 "hbm_frac_of_measured": round(byts / (us * 1e-6) / 1e9 / peak, 3),
                 "tflops": round(flops / (us * 1e-6) / 1e12, 1),
                 "weight_matrices_rotated": nmat}
            # the codes go to the tensor core as they are: the FP8 rate, twice the measured bf16 figure
            r["mma"] = ("kind::f8f6f4 (e4m3 x e4m3)" if fmt == "fp8" else
                        "kind::mxf8f6f4.block_scale (e2m1 x e4m3, e8m0 group scales in TMEM)") + ", no conversion"
            r["tensor_frac"] = round(flops / (us * 1e-6) / 1e12 / (2 * tf_peak), 3)
            r["tensor_peak_tflops"] = 2 * tf_peak
            # context: cuBLAS bf16 on pre-dequantized weights (same shape)
            if fmt == "fp8":
                wb = torch.empty((N, K), dtype=torch.bfloat16, device=dev)
                L.call("dsmoe_fp8_block_dequant", q.data_ptr(), sc.data_ptr(), N, K, 128, wb.data_ptr(),
                       L.DTYPE_BF16, st)
                xbf = x.to(torch.bfloat16)
                for _ in range(3):
                    torch.matmul(xbf, wb.T)
                torch.cuda.synchronize(dev)
                e0.record()
                for _ in range(args.steps):
                    torch.matmul(xbf, wb.T)
                e1.record()
                torch.cuda.synchronize(dev)
                r["cublas_bf16_us"] = round(e0.elapsed_time(e1) * 1e3 / args.steps, 2)
                r["cublas_bf16_note"] = "one weight matrix (L2-resident for M <= 126), bf16 x bf16"
                del wb
            res[f"{fmt}_m{M}"] = r
        del qs, scs
        torch.cuda.empty_cache()
    line = {"mode": "gemm", "metric": "kernel-surface fp8_gemm / fp4_gemm us per call (tcgen05)",
            "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "config": {"workload": "out[M, 5120] = (e4m3 a * a_s) @ dequant(W[5120, 5120])^T, bf16 out",
                       "M": [1, 126, 2048], "activations": "e4m3 + fp32 scale per 128-K block",
                       "l2": "weights rotate over > 3x L2 of distinct matrices"},
            "kernels": res, "peak_hbm_gbs": peak, "peak_source": peak_kind, "peak_bf16_tflops": tf_peak,
            "tensor_frac_note": "GEMM flops over 2x the measured bf16 peak (the dense FP8 rate)",
            "timing": "CUDA graph of back-to-back calls, CUDA events around the replays"}
    print(json.dumps(line), flush=True)


def sweep_mode(args):
    """Config: decode batch 1..64 on one FP8 and one FP4 layer (router routing, ~uniform), and the
    batched tcgen05 path under forced uniform and Zipf(1.1) routing at the same batches."""
    import torch
    import dsmoe
    from dsmoe import _lib as L
    from dsmoe.tp import env_rank_world
    rank, local, world = env_rank_world()
    if world != 1:
        raise SystemExit("--mode sweep runs on one GPU")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    layers, _ = build_layers(args, dev, 0, 1, layer_formats(args), max_tokens=64)
    gen = torch.Generator().manual_seed(args.seed + 2)
    pool = dsmoe.make_tokens(128, H, gen).to(dev)
    peak, _ = measured_peak()
    w13_b = {"fp8": FP8_W13, "fp4": FP4_W13}
    w2_b = {"fp8": FP8_W2, "fp4": FP4_W2}
    rows = []
    for B in (1, 2, 4, 8, 16, 32, 64):
        x = pool[:B].contiguous()
        outs = [torch.empty((B, H), dtype=torch.bfloat16, device=dev) for _ in layers]
        idxs = [torch.empty((B, TOPK), dtype=torch.int64, device=dev) for _ in layers]
        fns = [lambda m=m, y=y, ix=ix: L.call("dsmoe_moe_decode", m._layer, L.ptr(x), B, None, L.ptr(y), L.DTYPE_BF16,
                                                L.ptr(ix), None, None, L.ptr(m.workspace), m.workspace.numel(),
                                                L.stream_of(x))
               for m, y, ix in zip(layers, outs, idxs)]
        ms = graph_times(fns, args.steps, args.warmup, dev)
        for m in layers:
            m.check(B)
        for nm, t, ix in zip(layer_formats(args), ms, idxs):
            u = len(set(ix.flatten().tolist()))
            byts = args.experts * (H * 4 + 4) + u * (w13_b[nm] + w2_b[nm]) + FP8_W13 + FP8_W2
            rows.append({"path": "decode", "routing": "router", "fmt": nm, "batch": B, "us": round(t * 1e3, 2),
                         "us_per_token": round(t * 1e3 / B, 3), "unique_experts": u,
                         "gbs": round(byts / (t * 1e-3) / 1e9, 1), "hbm_frac": round(byts / (t * 1e-3) / 1e9 / peak, 3)})
        for rname, rfun in (("uniform", uniform_routing), ("zipf", dsmoe.zipf_routing)):
            idx, wt = rfun(B, args.experts, TOPK, gen)
            u = len(set(idx.flatten().tolist()))
            idx_d, wt_d = idx.to(dev), wt.to(dev)
            ms = graph_times([lambda m=m: m.prefill(x, idx_d, wt_d) for m in layers], args.steps, args.warmup, dev)
            for nm, t in zip(layer_formats(args), ms):
                byts = u * (w13_b[nm] + w2_b[nm]) + FP8_W13 + FP8_W2
                flops = 2.0 * 3 * H * I * (B * TOPK + B)
                rows.append({"path": "batched-tcgen05", "routing": rname, "fmt": nm, "batch": B,
                             "us": round(t * 1e3, 2), "us_per_token": round(t * 1e3 / B, 3), "unique_experts": u,
                             "gbs": round(byts / (t * 1e-3) / 1e9, 1),
                             "hbm_frac": round(byts / (t * 1e-3) / 1e9 / peak, 3),
                             "tflops": round(flops / (t * 1e-3) / 1e12, 2)})
    print(json.dumps({"mode": "sweep", "metric": METRIC, "unit": "us/layer", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "experts": args.experts, "peak_hbm_gbs": peak, "rows": rows}), flush=True)


def time_stack(layers, comm, dev, steps, warmup, seed):
    """One decode token (B = 1) through every layer, y of a layer being x of the next, as one CUDA
    graph (the MoE half of the reference's per-token DecodeTrace, dsv41/tt/model.py:262-446).
    Returns (ms per token, mean us per layer of the first half, of the second half), max over ranks:
    the time per token from a graph with events at its ends only (consecutive layer kernels overlap,
    programmatic dependent launch), the per-layer split from a second graph with events between layers."""
    import torch
    import torch.distributed as dist
    import dsmoe
    from dsmoe import _lib as L
    from dsmoe.tp import max_over_ranks
    B, nl = 1, len(layers)
    world = dist.get_world_size() if dist.is_initialized() else 1
    xs = [torch.empty((B, H), dtype=torch.bfloat16, device=dev) for _ in range(nl + 1)]
    idx = [torch.empty((B, TOPK), dtype=torch.int64, device=dev) for _ in range(nl)]
    tokpool = dsmoe.make_tokens(64, H, torch.Generator(device=dev).manual_seed(seed + 3), device=dev)

    def layer(li):
        m = layers[li]
        st_ = torch.cuda.current_stream(dev).cuda_stream
        if comm is not None:
            L.call("dsmoe_moe_decode_allreduce", m._layer, comm.handle, L.ptr(xs[li]), B, None, L.ptr(xs[li + 1]),
                   L.DTYPE_BF16, L.ptr(idx[li]), None, None, L.ptr(m.workspace), m.workspace.numel(), st_)
        else:
            L.call("dsmoe_moe_decode", m._layer, L.ptr(xs[li]), B, None, L.ptr(xs[li + 1]), L.DTYPE_BF16,
                   L.ptr(idx[li]), None, None, L.ptr(m.workspace), m.workspace.numel(), st_)

    if world > 1:
        dist.barrier()
        torch.cuda.synchronize(dev)
    xs[0].copy_(tokpool[:B])
    for li in range(nl):
        layer(li)
    torch.cuda.synchronize(dev)
    ev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(nl + 1)]
    pe = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(2)]
    g, gp = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for li in range(nl):
            ev[li].record()
            layer(li)
        ev[nl].record()
    with torch.cuda.graph(gp):
        pe[0].record()
        for li in range(nl):
            layer(li)
        pe[1].record()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    lt = [[] for _ in range(nl)]
    st = []
    for split in (False, True):
        for s in range(warmup + steps):
            xs[0].copy_(tokpool[s % 64:s % 64 + B])  # a new token each step
            (g if split else gp).replay()
            torch.cuda.synchronize(dev)
            if s >= warmup:
                if split:
                    for li in range(nl):
                        lt[li].append(ev[li].elapsed_time(ev[li + 1]))
                else:
                    st.append(pe[0].elapsed_time(pe[1]))
    for m in layers:
        m.check(B)
    del g, gp  # released before any process group goes away
    half = nl // 2
    ms_tok = max_over_ranks(statistics.mean(st), dev)
    a_us = max_over_ranks(statistics.mean(statistics.mean(lt[li]) for li in range(half)) * 1e3, dev)
    b_us = max_over_ranks(statistics.mean(statistics.mean(lt[li]) for li in range(half, nl)) * 1e3, dev)
    return ms_tok, a_us, b_us


def stack_from_layers(args, layers, comm, dev, rank, world, n_total):
    """Config 4 beside the decode line: ``n_total`` resident layers (first half FP8, second half FP4)
    at B = 1. The two benchmark layers are the first FP8 and FP4 layers; every other layer gets its
    own memory holding a copy of their expert bytes and its own seeded router, so each layer streams
    its own weights and routes differently. Built only when it fits in every rank's free memory."""
    import torch
    import torch.distributed as dist
    import dsmoe
    by_fmt = {m.fmt: m for m in layers}
    if set(by_fmt) != {"fp8", "fp4"}:
        return None
    per = {f: by_fmt[f].nbytes + by_fmt[f].workspace.numel() + 16e6 for f in by_fmt}
    need = (n_total // 2 - 1) * (per["fp8"] + per["fp4"])
    free, _ = torch.cuda.mem_get_info(dev)
    fits = torch.tensor([1 if need < free - 4e9 else 0], device=dev)
    if world > 1:
        dist.all_reduce(fits, op=dist.ReduceOp.MIN)
    if not bool(fits.item()):
        return {"skipped": f"{n_total} layers need {need / 1e9:.0f} GB more per GPU than is free"}
    t0 = time.time()
    gen = torch.Generator(device=dev).manual_seed(args.seed + 11)
    stack = []
    for fmt in ("fp8", "fp4"):
        src = by_fmt[fmt]
        for j in range(n_total // 2):
            if j == 0:
                stack.append(src)
                continue
            m = dsmoe.MoE(H, I, src.n_experts, TOPK, fmt, "sigmoid", ROUTE_SCALE, rank=rank, world=world, device=dev,
                          max_tokens=8, layouts=tuple(src.stores))
            m.load_router(dsmoe.make_router(src.n_experts, H, gen, device=dev))
            m.copy_experts_from(src)
            if comm is not None:
                m.use_comm(comm)
            stack.append(m)
    torch.cuda.synchronize(dev)
    build_s = time.time() - t0
    ms_tok, fp8_us, fp4_us = time_stack(stack, comm, dev, max(10, args.steps), max(3, args.warmup), args.seed)
    del stack
    torch.cuda.empty_cache()
    return {"ms_per_token": round(ms_tok, 4), "layers": n_total, "batch": 1,
            "layer_us": {"fp8": round(fp8_us, 2), "fp4": round(fp4_us, 2)},
            "weights": "layers 0 (FP8) and 20 (FP4) are the benchmark layers; the others hold copies of their expert "
                       "bytes in their own memory, each with its own seeded router",
            "timing": "CUDA events at the ends of one graph of all layers (y of a layer feeds the next), max over ranks",
            "build_s": round(build_s, 1)}


def stack_mode(args):
    """Config: the 40-layer MoE stack (layers 0-19 FP8, 20-39 FP4), decode batch 1, every layer's
    experts resident, each GPU holding 1/N of every expert, each layer ending in its all-reduce (in
    the layer kernel at N > 1). One token step is one CUDA graph of all layers, y of layer l being
    x of layer l + 1 (the MoE half of the reference's per-token DecodeTrace, dsv41/tt/model.py:262-446).
    With fewer GPUs than the stack needs, as many FP8 / FP4 layer pairs as fit are built."""
    import datetime
    import torch
    import torch.distributed as dist
    import dsmoe
    from dsmoe.tp import PeerComm, env_rank_world
    rank, local, world = env_rank_world()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    emu = args.emulate_tp if world == 1 else 1
    slices = world * emu  # expert slices: the layer is built as rank `rank` of `slices`
    per_pair = (E * (FP8_W13 + FP8_W2 + FP4_W13 + FP4_W2) + 2 * (FP8_W13 + FP8_W2)) / slices + 2 * (E * H * 4 + 64e6)
    free, _ = torch.cuda.mem_get_info(dev)
    pairs = min(args.stack_layers // 2, int((free - 6e9) // per_pair))
    if world > 1:  # every rank builds the same number of layers
        t = torch.tensor([pairs], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        pairs = int(t.item())
    if pairs < 1:
        raise SystemExit("not enough device memory for one FP8 + FP4 layer pair")
    fmts = ["fp8"] * pairs + ["fp4"] * pairs
    t0 = time.time()
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    layers = []
    for fmt in fmts:  # each layer its own uniform-random router and experts
        m = dsmoe.MoE(H, I, E, TOPK, fmt, "sigmoid", ROUTE_SCALE, rank=rank, world=slices, device=dev, max_tokens=8,
                      layouts=decode_layouts(1))
        m.load_router(dsmoe.make_router(E, H, gen, device=dev))
        m.load_shared(dsmoe.make_expert("fp8", H, I, gen, device=dev))
        for e in range(E):
            m.load_expert(e, dsmoe.make_expert(fmt, H, I, gen, device=dev))
        layers.append(m)
    comm = None
    if world > 1:
        comm = PeerComm(H, device=dev)
        for m in layers:
            m.use_comm(comm)
    setup_s = time.time() - t0
    nl = len(layers)
    ms_tok, fp8_us, fp4_us = time_stack(layers, comm, dev, args.steps, args.warmup, args.seed)
    if rank == 0:
        print(json.dumps({
            "mode": "stack", "metric": "MoE stack ms/token (decode batch 1, all experts resident)",
            "value": round(ms_tok, 4), "unit": "ms/token", "n_gpus": world, "layers": nl, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False,
            "ms_per_token_40_layers": round(ms_tok * 40 / nl, 4),
            "timing": "CUDA events at the ends of one graph of all layers (per-layer split from a second graph "
                      "with events between layers)",
            "layer_us": {"fp8": round(fp8_us, 2), "fp4": round(fp4_us, 2)},
            "config": {"workload": f"{nl}-layer MoE stack ({pairs} FP8 + {pairs} FP4 layers), y of a layer feeding "
                                   f"the next, one CUDA graph per token",
                       "parallelism": f"tp{world}" if emu == 1 else f"emulated tp{emu} on one GPU (rank 0's slice, no all-reduce)",
                       "allreduce": "in-kernel NVLink peer exchange" if world > 1 else None,
                       "experts": E, "hidden": H, "inter": I},
            "setup_s": round(setup_s, 1)}), flush=True)
    if world > 1:
        dist.barrier()
        comm.close()
        dist.destroy_process_group()


def main():
    global DECODE_STORE
    args = parse()
    DECODE_STORE = args.decode_store
    if args.impl == "reference":
        reference_arm(args)
    elif args.mode == "prefill":
        prefill_mode(args)
    elif args.mode == "sweep":
        sweep_mode(args)
    elif args.mode == "gemm":
        gemm_mode(args)
    elif args.mode == "stack":
        stack_mode(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
