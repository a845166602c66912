"""Benchmark of the b200 non-GEMM op path: the row-sharded Llama-3-8B-shaped stack.

Workload (one "step"): 32 decoder layers of the non-GEMM chain
  RMSNorm(hidden 4096, eps 1e-5) -> RoPE on q [T,32,128] / k [T,8,128]
  (theta 1e4, global positions) -> SwiGLU (intermediate 14336) -> residual add
over 131072 bf16 tokens split by rows across the ranks (no collective on the
hot path).  Activations ~ N(0,1), weights ~ 1 + N(0,0.1), per-layer weights
seeded 1000*layer + tensor id; one activation set per rank is reused by all
layers (the bytes moved are the same as with fresh activations per layer).

Outputs ONE JSON line (rank 0):
  value     tokens/s of the whole job, inputs resident in HBM, device time
            (CUDA events), max over ranks; the step is replayed as one CUDA
            graph of its launch list (--no-graph: eager launches).
  e2e       the same metric through the reference-facing plugin API (flagos
            tensors, torch_fl.ops) with the hidden state copied from pinned
            host memory before and back after every step.
  roofline  the kernel with the largest total time (SwiGLU) against the
            measured HBM copy bandwidth.
  gpu_eager_reference  the HF formulas on PyTorch's own CUDA kernels (what
            the reference's cuda route runs) on the same stack, N=1.
  per_op    achieved HBM GB/s of every kernel of the step (CUDA events
            around each launch, in a second timed pass of the same steps
            launched one by one).
  cpu_baseline  the reference's CPU path (HF formulas on torch CPU aten) on
            a bounded sample, rank 0 at N=1.

`--impl reference` times the reference's own CPU implementation of the path
(the same HF formulas on torch CPU aten, all host threads) on a bounded
sample and prints the same metric with "impl": "reference".
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "pytorch-plugin-fl_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

HIDDEN, HQ, HKV, HEAD, INTER = 4096, 32, 8, 128, 14336
EPS, THETA = 1e-5, 10000.0
BF16 = 2
# Algorithmic HBM bytes per token per layer (every input read once, every
# output written once):
BYTES = {
    "rms_norm": 2 * HIDDEN * BF16,                          # x in, out
    "rope_qk": 2 * (HQ + HKV) * HEAD * BF16,                # q,k in and out
    "swiglu": 3 * INTER * BF16,                             # gate, up in; act out
    "residual_add": 3 * HIDDEN * BF16,                      # x, y in; h out
}
BYTES["swiglu_residual"] = BYTES["swiglu"] + BYTES["residual_add"]
BYTES_PER_TOKEN_LAYER = BYTES["rms_norm"] + BYTES["rope_qk"] + BYTES["swiglu_residual"]
TABLE_BYTES_PER_TOKEN = 2 * HEAD * BF16                     # cos/sin rows (cached)

WORKLOAD = ("Llama-3-8B-shaped non-GEMM stack: 32 layers x [RMSNorm(4096) -> RoPE(q 32x128, "
            "k 8x128) -> SwiGLU(14336) -> residual add], bf16, tokens split by rows")


def _env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic():
    """Per-token DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/traffic.json), or None."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return None


class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled during the timed
    region: NVML polled from a thread every 10 ms (read-only queries), so a
    timed region of ~0.1 s still gets samples; nvidia-smi every 200 ms when
    NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        # NVML and nvidia-smi number GPUs physically; map through CUDA_VISIBLE_DEVICES.
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        self.gpu = int(ids[gpu_index]) if gpu_index < len(ids) and ids[gpu_index].isdigit() \
            else gpu_index
        self.samples = []
        self.thread = None
        self.proc = None
        self.path = os.path.join("/tmp", f"fl_b200_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            import threading

            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            smax = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            masks = [(n, getattr(pynvml, c)) for n, c in self.REASONS]
            self.stop_flag = threading.Event()

            def poll():
                while not self.stop_flag.is_set():
                    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((sm, smax, [n for n, m in masks if bits & m]))
                    self.stop_flag.wait(0.01)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            if not self.samples:
                return None
            sm = [s[0] for s in self.samples]
            reasons = sorted({r for s in self.samples for r in s[2]})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(s[1] for s in self.samples),
                    "reasons": reasons, "samples": len(self.samples), "source": "nvml 10 ms"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        try:
            os.remove(self.path)
        except OSError:
            pass
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi 200 ms"}


def rope_tables(pos0, T, device):
    """bf16 cos/sin [T, 128] for global positions pos0..pos0+T-1, built as
    Qwen3RotaryEmbedding builds them (inv_freq = 1/theta^(arange(0,D,2)/D),
    fp32 position product, cat, cos/sin, cast) on torch CPU, then copied to
    the device: the table is then HF's CPU table bit for bit."""
    pos = torch.arange(pos0, pos0 + T, dtype=torch.int64).to(torch.float32)
    inv = 1.0 / (THETA ** (torch.arange(0, HEAD, 2, dtype=torch.int64).to(torch.float32) / HEAD))
    fr = pos[:, None] * inv[None, :]
    emb = torch.cat([fr, fr], dim=-1)
    return (emb.cos().to(torch.bfloat16).to(device), emb.sin().to(torch.bfloat16).to(device))


# ---------------------------------------------------------------- the stack
class Stack:
    """Device-resident buffers of one rank's row shard and the launch list."""

    def __init__(self, tokens, layers, pos0, device, rounding, fuse_add_norm):
        from torch_fl import kernels as K

        self.K = K
        self.T, self.L, self.dev = tokens, layers, device
        self.rounding = rounding
        self.fuse = fuse_add_norm
        rank = _env_int("RANK", 0)
        g = torch.Generator(device=device)

        def rn(seed, *shape, scale=1.0, loc=0.0, per_rank=True):
            # activations: the rank's own rows; weights: the same on every rank
            g.manual_seed(seed + (100000 * rank if per_rank else 0))
            return (loc + scale * torch.randn(*shape, generator=g, device=device)).to(torch.bfloat16)

        T = tokens
        self.x0 = rn(1, T, HIDDEN)
        self.q = rn(2, 1, T, HQ, HEAD)
        self.k = rn(3, 1, T, HKV, HEAD)
        self.g = rn(4, T, INTER)
        self.u = rn(5, T, INTER)
        self.y = rn(6, T, HIDDEN)
        self.w = [rn(1000 * l + 7, HIDDEN, scale=0.1, loc=1.0, per_rank=False)
                  for l in range(layers)]
        self.cos, self.sin = rope_tables(pos0, T, device)
        self.pos0 = pos0
        # outputs (reused by every layer)
        self.xa = torch.empty_like(self.x0)
        self.xb = torch.empty_like(self.x0)
        self.n = torch.empty_like(self.x0)
        self.qo = torch.empty_like(self.q)
        self.ko = torch.empty_like(self.k)
        self.a = torch.empty_like(self.g)

    def launches_per_step(self):
        return (3 * self.L + 1) if self.fuse else 3 * self.L

    def run(self, x_in, timer=None):
        """One step over all layers; returns the final hidden state buffer.
        timer(name) returns a context manager that brackets one launch."""
        K, r = self.K, self.rounding
        x, nxt = x_in, self.xa
        def t(name):
            return timer(name) if timer else _null
        if self.fuse:
            with t("rms_norm"):
                K.rms_norm(x, self.w[0], EPS, rounding=r, out=self.n)
        for l in range(self.L):
            if not self.fuse:
                with t("rms_norm"):
                    K.rms_norm(x, self.w[l], EPS, rounding=r, out=self.n)
            with t("rope_qk"):
                self._rope()
            if self.fuse and l + 1 < self.L:
                with t("swiglu"):
                    K.swiglu(self.g, self.u, rounding=r, out=self.a)
                with t("add_rms_norm"):
                    K.add_rms_norm(x, self.y, self.w[l + 1], EPS, rounding=r, h_out=nxt, out=self.n)
            else:
                with t("swiglu_residual"):
                    K.swiglu_residual(self.g, self.u, x, self.y, rounding=r, act_out=self.a, h_out=nxt)
            x, nxt = nxt, (self.xb if nxt is self.xa else self.xa)
        return x

    # ---- the same stack through the public plugin API on flagos tensors ----
    def flagos_views(self):
        """Zero-copy flagos views of the rank's buffers (flagos memory is
        CUDA memory of the same GPU)."""
        from torch_fl import _C

        v = _C._cuda_to_flagos_view
        self.fq, self.fk, self.fg, self.fu, self.fy = (v(t) for t in (self.q, self.k, self.g,
                                                                      self.u, self.y))
        self.fcos, self.fsin = v(self.cos), v(self.sin)
        self.fw = [v(w) for w in self.w]

    def run_flagos(self, x, rows=None):
        """One step through torch_fl.ops (flagos:: ops through PyTorch's
        dispatcher, outputs allocated by the flagos allocator) over the
        tokens `rows` (a slice; all tokens when None).  Every op of the stack
        is per token, so a token chunk runs the same 32 layers on its rows."""
        import torch_fl.ops as O

        s = slice(None) if rows is None else rows
        fq, fk, fg, fu, fy = self.fq[:, s], self.fk[:, s], self.fg[s], self.fu[s], self.fy[s]
        fcos, fsin = self.fcos[s], self.fsin[s]
        r = self.rounding
        n = O.rms_norm(x, self.fw[0], EPS, r)
        for l in range(self.L):
            qo, ko = O.rope_qk(fq, fk, fcos, fsin, 2, r)
            if l + 1 < self.L:
                a = O.swiglu(fg, fu, r)
                n, x = O.add_rms_norm(x, fy, self.fw[l + 1], EPS, r)
            else:
                a, x = O.swiglu_residual(fg, fu, x, fy, r)
        return x

    def run_torch_eager(self, x, layers):
        """`layers` layers of the HF formulas on PyTorch's own CUDA kernels
        (the kernels the reference's cuda route runs): RMSNorm
        (modeling_qwen3.py:59-64), apply_rotary_pos_emb (:158-181),
        silu(gate) * up (:81-82), residual add."""
        q = self.q.transpose(1, 2)        # [B, H, S, D] view, as HF passes it
        k = self.k.transpose(1, 2)
        cos, sin = self.cos[None, None], self.sin[None, None]

        def rotate_half(t):
            return torch.cat((-t[..., HEAD // 2:], t[..., :HEAD // 2]), dim=-1)

        for l in range(layers):
            h = x.to(torch.float32)
            h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + EPS)
            n = self.w[l] * h.to(x.dtype)
            qe = (q * cos) + (rotate_half(q) * sin)
            ke = (k * cos) + (rotate_half(k) * sin)
            a = torch.nn.functional.silu(self.g) * self.u
            x = x + self.y
        return x, n, qe, ke, a

    def _rope(self):
        self.K.rope_qk(self.q, self.k, self.cos, self.sin, layout="bshd", rounding=self.rounding,
                       q_out=self.qo, k_out=self.ko)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


_null = _Null()


class EventTimer:
    """Brackets launches with CUDA events on the current stream."""

    def __init__(self):
        self.ev = {}

    def __call__(self, name):
        timer = self

        class _Ctx:
            def __enter__(self_):
                self_.s = torch.cuda.Event(enable_timing=True)
                self_.e = torch.cuda.Event(enable_timing=True)
                self_.s.record()
                return self_

            def __exit__(self_, *a):
                self_.e.record()
                timer.ev.setdefault(name, []).append((self_.s, self_.e))
                return False

        return _Ctx()

    def mean_ms(self):
        return {k: sum(s.elapsed_time(e) for s, e in v) / len(v) for k, v in self.ev.items()}

    def counts(self):
        return {k: len(v) for k, v in self.ev.items()}


# ----------------------------------------------------------- CPU reference
def cpu_reference(sample_tokens, reps, threads, warmup=1):
    """The reference's own CPU path on a bounded sample: one decoder layer's
    chain on `sample_tokens` tokens, HF formulas over torch CPU aten.  Returns
    (seconds per token-layer, description, median ms of one sample)."""
    from oracle import hf_chain

    torch.set_num_threads(threads)
    T = sample_tokens
    g = torch.Generator().manual_seed(0)
    bf = torch.bfloat16

    def rn(*s, scale=1.0, loc=0.0):
        return (loc + scale * torch.randn(*s, generator=g)).to(bf)

    x, y, w = rn(T, HIDDEN), rn(T, HIDDEN), rn(HIDDEN, scale=0.1, loc=1.0)
    q = rn(1, T, HQ, HEAD).transpose(1, 2)
    k = rn(1, T, HKV, HEAD).transpose(1, 2)
    gt, up = rn(T, INTER), rn(T, INTER)
    cos, sin = hf_chain.rope_tables(torch.arange(T)[None], HEAD, THETA, bf)
    for _ in range(max(warmup, 1)):
        hf_chain.decoder_chain(x, w, q, k, cos, sin, gt, up, y, EPS)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        hf_chain.decoder_chain(x, w, q, k, cos, sin, gt, up, y, EPS)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    desc = (f"HF formulas (modeling_qwen3.py RMSNorm/apply_rotary_pos_emb/silu*up) + add on torch "
            f"{torch.__version__} CPU aten, one decoder layer x {T} tokens, median of {reps}; "
            f"extrapolated to the 32-layer stack by tokens x layers")
    return med / T, desc, med * 1e3


def cpu_info():
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return model


def capture_graph(fn):
    """Capture `fn`'s launches as a CUDA graph (one warm-up run on a side
    stream first, as torch.cuda.graph requires)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        fn()
    torch.cuda.synchronize()
    return gr


def workload_config(args, world):
    """The workload both arms run (the same dict on the b200 and the
    reference line)."""
    return {"workload": WORKLOAD, "tokens": args.tokens, "tokens_per_rank": args.tokens // world,
            "layers": args.layers, "hidden": HIDDEN, "intermediate": INTER,
            "heads": [HQ, HKV, HEAD], "parallelism": f"rows/{world}",
            "l2": "inputs larger than L2 (every per-rank activation >= 256 MB)"}


# --------------------------------------------------------------------- main
def default_e2e_chunks(world):
    """Token chunks per e2e step.  One rank: 2 (measured on B200, 88.1 ms per
    step against 89.7 with 4 -- more launches and kernel tails -- and 117
    with 1)."""
    return 2


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--tokens", type=int, default=131072)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--rounding", default="fused", choices=["fused", "chain"])
    ap.add_argument("--no-fuse-add-norm", action="store_true")
    # one layer of the 8192-token chain: the rate per token of a smaller,
    # cache-resident sample is higher (2048 tokens: 1.7x on one host)
    ap.add_argument("--cpu-sample-tokens", type=int, default=8192)
    ap.add_argument("--cpu-reps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunks", type=int, default=0,
                    help="token chunks per e2e step: host->device copies, the layers and the "
                         "device->host copies of different chunks overlap on three flagos "
                         "streams (0: the per-N default)")
    ap.add_argument("--e2e-sweep", default="",
                    help="comma-separated chunk counts to time after the e2e measurement "
                         "(reported as ms_per_step_by_chunks)")
    ap.add_argument("--no-eager", action="store_true")
    ap.add_argument("--no-hf-e2e", action="store_true",
                    help="skip the HF decoder-model leg (hidden states host -> flagos -> host)")
    ap.add_argument("--eager-layers", type=int, default=4)
    ap.add_argument("--no-op-configs", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="time the headline with eager launches instead of a CUDA graph replay")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch without programmatic dependent launch (the default uses it)")
    ap.add_argument("--profile-case", choices=sorted(PROFILE_CASES),
                    help="run one small case of one op once on GPU 0 and exit (for ncu)")
    ap.add_argument("--op-configs-only", action="store_true",
                    help="time only the per-op configurations on GPU 0 and print them")
    ap.add_argument("--case", default=None,
                    help="regular expression: time only the per-op configurations it matches")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case)
        return
    if args.op_configs_only:
        import torch_fl  # noqa: F401
        from torch_fl import _abi

        _abi.set_pdl(not args.no_pdl)
        torch.cuda.set_device(0)
        print(json.dumps({"per_op_configs": op_configs(torch.device("cuda", 0),
                                                       measured_peak()[0], only=args.case)}))
        return
    assert args.warmup >= 3 or os.environ.get("FL_B200_BENCH_ALLOW_SHORT"), "use --warmup >= 3"

    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    local = _env_int("LOCAL_RANK", 0)
    threads = os.cpu_count() or 1

    if args.impl == "reference":
        if rank != 0:
            return
        reps = max(args.steps, 1)
        per, desc, sample_ms = cpu_reference(args.cpu_sample_tokens, reps, threads,
                                             warmup=args.warmup)
        value = 1.0 / (per * args.layers)
        # Each step times one decoder layer of the chain on `sample_tokens`
        # tokens (BASELINE's 8192-token chain by default); the stack's rate is
        # that per-token-layer time scaled to `layers` layers.  ms_per_step is
        # the time of the step actually run; the full stack's time per step
        # is given under its own key.
        line = {"metric": "fused-layer tokens/s", "value": value, "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": sample_ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "impl": "reference", "extrapolated": True,
                "sample_tokens": args.cpu_sample_tokens, "sample_layers": 1,
                "sample_ms_median": sample_ms,
                "ms_per_step_extrapolated": per * args.tokens * args.layers * 1e3,
                "config": workload_config(args, world),
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                                 "kind": "reference", "sample": desc, "cpu": cpu_info()},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch_fl  # noqa: F401  (loads libfl_b200.so; fails loudly if missing)
    from torch_fl import _abi
    from torch_fl import kernels as K
    from torch_fl import sharding

    _abi.set_pdl(not args.no_pdl)

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        # The rank's GPU is current; no device_id (torch_fl makes flagos the
        # current accelerator, and NCCL binds to the current CUDA device).
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    T = args.tokens // world
    assert T * world == args.tokens, "tokens must split evenly across ranks"
    stack = Stack(T, args.layers, rank * T, dev, args.rounding, not args.no_fuse_add_norm)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            import torch.distributed as dist

            # an all-reduce on the rank's own GPU: no device inference involved
            dist.all_reduce(torch.zeros(1, device=dev))
        torch.cuda.synchronize()

    # warm-up
    for _ in range(args.warmup):
        stack.run(stack.x0)
    barrier()

    # The step's launch list captured once as a CUDA graph: a replay issues
    # the same kernels on the same buffers without per-launch host work.
    graph = None
    if not args.no_graph:
        graph = capture_graph(lambda: stack.run(stack.x0))
        for _ in range(args.warmup):
            graph.replay()
        barrier()
    step = graph.replay if graph is not None else (lambda: stack.run(stack.x0))

    # timed region (the headline): device time with events on the launching
    # stream, max over ranks
    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    barrier()
    clock_info = clocks.stop()
    ms = sharding.max_over_ranks(start.elapsed_time(end), dev)
    ms_per_step = ms / args.steps
    value = args.tokens * args.steps / (ms / 1e3)

    # A/B of programmatic dependent launch: the same step captured with
    # the opposite setting, timed the same way (every rank takes it).
    pdl_ab = None
    if graph is not None:
        _abi.set_pdl(args.no_pdl)
        g_ab = capture_graph(lambda: stack.run(stack.x0))
        _abi.set_pdl(not args.no_pdl)
        for _ in range(args.warmup):
            g_ab.replay()
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(args.steps):
            g_ab.replay()
        a1.record()
        torch.cuda.synchronize()
        barrier()
        ab_ms = sharding.max_over_ranks(a0.elapsed_time(a1), dev)
        del g_ab
        pdl_ab = {"pdl": args.no_pdl, "ms_per_step": ab_ms / args.steps,
                  "value": args.tokens * args.steps / (ab_ms / 1e3),
                  "what": "the same graph step captured with programmatic dependent launch "
                          + ("on" if args.no_pdl else "off")}

    # Per-kernel durations: a second timed pass of the same steps launched
    # one by one with CUDA events around every launch (the events would add
    # their own cost to the headline, so they are kept out of it).
    timer = EventTimer()
    barrier()
    pass_start, pass_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pass_start.record()
    for _ in range(args.steps):
        stack.run(stack.x0, timer)
    pass_end.record()
    torch.cuda.synchronize()
    barrier()
    timed_pass_ms = sharding.max_over_ranks(pass_start.elapsed_time(pass_end), dev) / args.steps
    if graph is not None:
        del graph  # release before the process group goes away

    kern_ms = timer.mean_ms()
    counts = timer.counts()
    per_op = {}
    bytes_of = dict(BYTES)
    bytes_of["add_rms_norm"] = 4 * HIDDEN * BF16
    for name, m in kern_ms.items():
        b = bytes_of[name] * T
        per_op[name] = {"ms": round(m, 4), "gbs": round(b / (m * 1e-3) / 1e9, 1),
                        "launches": counts[name]}
    # the dominant kernel: the largest total device time inside the timed region
    dom = max(kern_ms, key=lambda k: kern_ms[k] * counts[k])
    dom_bytes = bytes_of[dom] * T
    achieved = dom_bytes / (kern_ms[dom] * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    traffic = None
    tj = committed_traffic()
    if tj and dom in tj.get("bytes_per_token", {}):
        traffic = tj["bytes_per_token"][dom] * T
    roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback", "unit": "GB/s", "frac": round(achieved / peak, 4),
                "traffic": traffic, "algorithmic_bytes": dom_bytes}

    # End to end through the reference-facing plugin API: the hidden state
    # comes from pinned host memory into flagos tensors, the 32 layers run as
    # torch_fl.ops (flagos:: ops through PyTorch's dispatcher, outputs from
    # the flagos allocator), the result goes back to pinned host memory; all
    # inside the timed region.  The step is cut into token chunks: chunk c's
    # host->device copy (stream `h2d`), its layers (the current stream) and
    # its device->host copy (stream `d2h`) are ordered by flagos events, so
    # PCIe traffic in both directions overlaps the layers of other chunks.
    e2e = None
    if not args.no_e2e:
        import torch_fl.flagos as flagos

        fdev = torch.device("flagos", local)
        stack.flagos_views()
        h_in = torch.empty(T, HIDDEN, dtype=torch.bfloat16, pin_memory=True)
        h_in.copy_(stack.x0)
        h_out = torch.empty_like(h_in, pin_memory=True)
        comp = flagos.current_stream(local)
        h2d, d2h = flagos.Stream(local), flagos.Stream(local)

        def run_e2e(chunks):
            """Times args.steps e2e steps cut into `chunks` token chunks:
            (ms for all steps, ms per step of each half, warm-up steps,
            host issue ms per step), max over ranks."""
            chunks = max(1, min(chunks, T))
            bounds = [(T * c // chunks, T * (c + 1) // chunks) for c in range(chunks)]
            # At most two steps in flight: the host waits for step s-2's last
            # device->host copy before queueing step s, as a serving loop bounds
            # its queue (device memory then stays at two steps' buffers).
            inflight = []
            host_s = [0.0]   # host time spent issuing steps (not waiting on `inflight`)

            def e2e_step():
                t_issue = time.perf_counter()
                for lo, hi in bounds:
                    with flagos.stream(h2d):
                        x_d = h_in[lo:hi].to(fdev, non_blocking=True)
                        landed = flagos.Event()
                        landed.record(h2d)
                    comp.wait_event(landed)
                    x_d.record_stream(comp)
                    res = stack.run_flagos(x_d, slice(lo, hi))
                    done = flagos.Event()
                    done.record(comp)
                    d2h.wait_event(done)
                    with flagos.stream(d2h):
                        h_out[lo:hi].copy_(res, non_blocking=True)
                    res.record_stream(d2h)
                ev = flagos.Event()
                ev.record(d2h)
                inflight.append(ev)
                host_s[0] += time.perf_counter() - t_issue
                if len(inflight) > 2:
                    inflight.pop(0).synchronize()

            # Warm-up until the flagos allocator's pool has settled: its blocks
            # are reused only on the stream that freed them and the steps in
            # flight hold blocks on three streams, so it grows for a while (on
            # B200 from 8 to about 18 steps, run to run; a step that grows it is
            # slow on the host).  At least `warmup` and 12 steps, then until
            # three steps in a row leave the pool's reserved bytes unchanged
            # (at most 40).
            def reserved():  # host-side counter: no synchronisation (steps stay in flight)
                return flagos.memory_stats().get("pool_reserved", 0)

            warm, still, last = 0, 0, -1
            with torch.inference_mode():
                while warm < 40 and (warm < max(args.warmup, 12) or still < 3):
                    e2e_step()
                    warm += 1
                    now = reserved()
                    pool_warm.append(now)
                    still = still + 1 if now == last else 0
                    last = now
            comp.wait_stream(d2h)
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            em = torch.cuda.Event(enable_timing=True)
            host_s[0] = 0.0
            marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            hmarks = []
            e0.record(comp)
            t0 = time.perf_counter()
            with torch.inference_mode():
                for i in range(args.steps):
                    e2e_step()
                    marks[i].record(comp)  # step i's layers are done at marks[i]
                    hmarks.append(time.perf_counter() - t0)  # step i queued on the host
                    pool_timed.append(reserved())
                    if i == args.steps // 2 - 1:
                        em.record(comp)    # the first half's layers are queued before em
            comp.wait_stream(d2h)          # the last chunk is in host memory at e1
            e1.record(comp)
            torch.cuda.synchronize()
            ems = sharding.max_over_ranks(e0.elapsed_time(e1), dev)
            # device time from the start to each step's last layer (max over ranks)
            each[:] = [round(sharding.max_over_ranks(e0.elapsed_time(m), dev), 3) for m in marks]
            heach[:] = [round(sharding.max_over_ranks(h * 1e3, dev), 3) for h in hmarks]
            halves = [ems / args.steps] * 2
            if args.steps >= 2:
                halves = [sharding.max_over_ranks(e0.elapsed_time(em), dev) / (args.steps // 2),
                          sharding.max_over_ranks(em.elapsed_time(e1), dev)
                          / (args.steps - args.steps // 2)]
            host_ms = sharding.max_over_ranks(host_s[0] * 1e3, dev) / args.steps
            return ems, halves, warm, host_ms

        chunks = max(1, min(args.e2e_chunks or default_e2e_chunks(world), T))
        each, heach, pool_warm, pool_timed = [], [], [], []
        ems, halves, warm, host_ms = run_e2e(chunks)
        # (warm-up: this rank's, its length differs by rank; timed: max over ranks)
        pool_mb = {"warm_up": [round(v / 2**20) for v in pool_warm],
                   "timed": [round(sharding.max_over_ranks(v, dev) / 2**20) for v in pool_timed]}
        layers_done_ms, queued_ms = list(each), list(heach)
        by_chunks = {}
        for c in sorted({int(v) for v in args.e2e_sweep.split(",") if v}):
            by_chunks[c] = round(run_e2e(c)[0] / args.steps, 3)
        # the e2e result equals the device-resident path's result
        same = bool(torch.equal(h_out.to(dev), stack.run(stack.x0)))
        nbytes = h_in.numel() * h_in.element_size()
        # This box's plain pinned-copy rates, one direction at a time, after
        # the timed region (the e2e step moves nbytes each way, so these set
        # its floor: measured 1.48 M tokens/s on one box and 0.87 M on
        # another with the same build and the same device-resident step).
        tmp = torch.empty_like(stack.x0)
        rates = {}
        for name, dst, src in (("h2d", tmp, h_in), ("d2h", h_out, tmp)):
            best = float("inf")
            for _ in range(2):
                c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                c0.record()
                dst.copy_(src, non_blocking=True)
                c1.record()
                torch.cuda.synchronize()
                best = min(best, c0.elapsed_time(c1))
            rates[name] = round(nbytes / (best / 1e3) / 1e9, 1)
        # The floor the host sets: one step's copy in and copy out running at
        # the same time on their two streams, every rank at once (as in the
        # e2e step).  With many ranks sharing the host's links and memory,
        # this, not the GPU, can bound the e2e step.
        tmp2 = torch.empty_like(stack.x0)
        barrier()
        floor = float("inf")
        for _ in range(2):
            f0 = torch.cuda.Event(enable_timing=True)
            f1 = torch.cuda.Event(enable_timing=True)
            f2 = torch.cuda.Event(enable_timing=True)
            f0.record(comp)
            h2d.wait_event(f0)
            d2h.wait_event(f0)
            with flagos.stream(h2d):
                tmp.copy_(h_in, non_blocking=True)
            with flagos.stream(d2h):
                h_out.copy_(tmp2, non_blocking=True)
            f1.record(h2d)
            f2.record(d2h)
            torch.cuda.synchronize()
            floor = min(floor, max(f0.elapsed_time(f1), f0.elapsed_time(f2)))
        floor = sharding.max_over_ranks(floor, dev)
        del tmp, tmp2
        e2e = {"value": args.tokens * args.steps / (ems / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": nbytes * world, "d2h_bytes_per_step": nbytes * world,
               "ms_per_step": ems / args.steps, "matches_device_path": same,
               "chunks": chunks, "host_copy_gbs": rates,
               "ms_per_step_halves": [round(h, 3) for h in halves],
               **({"ms_per_step_by_chunks": by_chunks} if by_chunks else {}),
               "layers_done_ms": layers_done_ms,
               "host_queued_ms": queued_ms,
               "pool_reserved_mb_after_each_step": pool_mb,
               "warmup_steps": warm,
               "copy_floor_ms": round(floor, 3),
               "host_issue_ms_per_step": round(host_ms, 3),
               "copy_floor_what": "one step's host->device and device->host copies at the same "
                                  "time on two streams, all ranks at once (max over ranks)",
               "api": "torch_fl.ops (flagos:: ops) on flagos tensors under "
                      "torch.inference_mode, host<->flagos copies on flagos streams "
                      "overlapping the layers"}

    # A real HF model through the public API: hidden states from pinned host
    # memory into a Llama-3-8B-shaped decoder (HF's own modules on flagos),
    # the last hidden state back, with the fused-op hooks on and off;
    # informational (the GEMMs dominate), N=1 only.
    e2e_hf = None
    if not args.no_hf_e2e and world == 1:
        e2e_hf = hf_model_e2e(dev, args)

    # PyTorch's own CUDA kernels on the HF formulas (the kernels the
    # reference's cuda route runs), same stack, `eager_layers` layers timed
    # and scaled to the full depth; informational.
    eager = None
    if not args.no_eager and world == 1:
        L = min(args.eager_layers, args.layers)
        for _ in range(2):
            stack.run_torch_eager(stack.x0, L)
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(2):
            stack.run_torch_eager(stack.x0, L)
        g1.record()
        torch.cuda.synchronize()
        ms_layer = g0.elapsed_time(g1) / (2 * L)
        eager = {"value": T / (ms_layer * args.layers / 1e3), "unit": "tokens/s",
                 "ms_per_layer": ms_layer, "layers_timed": L,
                 "what": f"HF formulas on torch {torch.__version__} CUDA eager kernels, bf16"}

    # correctness gather (NCCL, outside the timed region): sampled rows of
    # every rank checked on rank 0 against the oracle
    check = correctness_sample(stack, K, world, rank, dev)

    per_op_configs = None
    if world == 1 and not args.no_op_configs:
        del stack.g, stack.u, stack.a        # room for the 17 GB softmax config
        torch.cuda.empty_cache()
        per_op_configs = op_configs(dev, measured_peak()[0], only=args.case)

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            per, desc, _ = cpu_reference(args.cpu_sample_tokens, args.cpu_reps, threads)
            cpu = {"value": 1.0 / (per * args.layers), "unit": "tokens/s", "cores": threads,
                   "kind": "reference", "sample": desc, "cpu": cpu_info()}
        line = {
            "metric": "fused-layer tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(args, world),
            "impl_config": {"rounding": args.rounding,
                            "fused_add_rms_norm": not args.no_fuse_add_norm,
                            "pdl": not args.no_pdl,
                            "launch": "CUDA graph replay of the step" if not args.no_graph
                                      else "eager launches"},
            "hbm_gbs_step": round(stack_bytes(stack) * args.steps / (ms / 1e3) / 1e9, 1),
            "per_op": per_op, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "pdl_ab": pdl_ab, "e2e_hf": e2e_hf,
            "gpu_eager_reference": eager, "per_op_configs": per_op_configs,
            "gpu_launches": stack.launches_per_step() * args.steps,
            "per_kernel_pass_ms_per_step": round(timed_pass_ms, 3),
            "clocks": clock_info, "correctness": check,
        }
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def hf_model_e2e(dev, args, layers=2, batch=4, seq=2048, steps=5):
    """transformers' LlamaModel (Llama-3-8B shapes: hidden 4096, 32 / 8 heads
    of 128, intermediate 14336, eps 1e-5, theta 1e4, eager attention) with
    `layers` random-init bf16 decoder layers on flagos.  One step: the
    [batch, seq, 4096] hidden states copied from pinned host memory, the
    forward (causal), the last hidden state copied back to pinned host
    memory; device time per step (CUDA events), with the fused-op hooks
    (torch_fl.enable_hf_fused_ops) and without them (HF's op chain on the
    flagos aten routes)."""
    import torch_fl
    from transformers import LlamaConfig, LlamaModel

    cfg = LlamaConfig(vocab_size=128, hidden_size=HIDDEN, intermediate_size=INTER,
                      num_hidden_layers=layers, num_attention_heads=HQ, num_key_value_heads=HKV,
                      head_dim=HEAD, max_position_embeddings=seq, rms_norm_eps=EPS,
                      rope_parameters={"rope_type": "default", "rope_theta": THETA},
                      attn_implementation="eager")
    torch.manual_seed(0)
    fdev = torch.device("flagos", dev.index)
    model = LlamaModel(cfg).to(torch.bfloat16).to(fdev).eval()   # ~6 s of CPU init
    g = torch.Generator().manual_seed(3)
    h_in = torch.randn(batch, seq, HIDDEN, generator=g).to(torch.bfloat16).pin_memory()
    h_out = torch.empty_like(h_in).pin_memory()

    def step():
        x = h_in.to(fdev, non_blocking=True)
        y = model(inputs_embeds=x).last_hidden_state
        h_out.copy_(y, non_blocking=True)

    res = {}
    outs = {}
    for hooks in (True, False):
        if hooks:
            torch_fl.enable_hf_fused_ops()
        with torch.no_grad():
            for _ in range(2):
                step()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                step()
            e1.record()
            torch.cuda.synchronize()
        outs[hooks] = h_out.clone()
        torch_fl.disable_hf_fused_ops()
        ms = e0.elapsed_time(e1) / steps
        res["hooks_on" if hooks else "hooks_off"] = {
            "ms_per_step": round(ms, 3), "tokens_per_s": round(batch * seq / (ms / 1e3), 1)}
    a, b = outs[True].float(), outs[False].float()
    res["max_abs_diff_on_vs_off"] = round((a - b).abs().max().item(), 5)
    res["max_abs_out"] = round(b.abs().max().item(), 3)
    res.update({"model": f"transformers LlamaModel, {layers} decoder layers of Llama-3-8B shape, "
                         "random init, bf16, eager attention", "batch": batch, "seq": seq,
                "h2d_bytes_per_step": h_in.numel() * 2, "d2h_bytes_per_step": h_out.numel() * 2})
    del model
    torch.cuda.empty_cache()
    return res


def op_configs(dev, peak, reps=5, only=None):
    """Per-op HBM GB/s on the other benchmark configurations (device time,
    CUDA events, median of `reps` after 2 warm-ups; inputs resident, each
    larger than L2 except the 67 MB RMSNorm f32 config, which L2 holds)."""
    from torch_fl import kernels as K

    out = {}
    g = torch.Generator(device=dev).manual_seed(7)

    # A case whose inputs L2 could hold gets an L2 flush before every timed
    # rep: 256 MB written, then another 256 MB read, so that L2 holds clean
    # lines of neither the case's inputs nor dirty flush data (whose
    # write-back would otherwise land inside the timed kernel).
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    flush_sink = torch.empty((), dtype=torch.float32, device=dev)

    import re

    def timed(name, fn, nbytes, note="", flush=False, tokens=None, reps_=None):
        if only and not re.search(only, name):
            return
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps_ or reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if flush:
                flush_buf.fill_(1)
                torch.sum(flush_rd, dim=0, out=flush_sink)
            # A bounded spin kernel keeps the GPU busy while the host prepares
            # the launch, so the events bracket the op's device time only.
            torch.cuda._sleep(2_000_000)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        ms = statistics.median(ts)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                     "bytes": int(nbytes)}
        if tokens:
            out[name]["tokens_per_s"] = round(tokens / (ms * 1e-3), 1)
        if flush:
            out[name]["l2"] = "flushed before each rep (256 MB written, then 256 MB read)"
        if note:
            out[name]["note"] = note

    def want(*names):
        return only is None or any(re.search(only, n) for n in names)

    if want("llama_chain_T8192", "rms_norm_bf16_8192x4096", "rope_qk_bf16_T8192",
            "swiglu_bf16_8192x14336", "add_bf16_8192x4096", "rms_norm_rope_bf16_T8192",
            "rms_norm_rope_bf16_T131072"):
        chain_configs(dev, g, timed)

    # config 1: RMSNorm fp32 [2048, 4096], eps 1e-6
    x = torch.randn(2048, 4096, generator=g, device=dev)
    w = 1 + 0.1 * torch.randn(4096, generator=g, device=dev)
    timed("rms_norm_f32_2048x4096", lambda: K.rms_norm(x, w, 1e-6), 2 * x.numel() * 4 + 4096 * 4,
          "67 MB: fits in L2")
    del x, w
    # config 3: causal softmax
    for dt, L, name in ((torch.bfloat16, 2048, "bf16_8x32x2048x2048"),
                        (torch.float16, 4096, "f16_8x32x4096x4096")):
        if not want(f"softmax_{name}", f"causal_softmax_{name}", f"softmax_{name}_f32_out",
                    f"masked_softmax_{name}", f"masked_softmax_{name}_torch_chain"):
            continue
        lg = (3.0 * torch.randn(8, 32, L, L, generator=g, device=dev)).to(dt)
        masked = lg.masked_fill(torch.triu(torch.ones(L, L, dtype=torch.bool, device=dev), 1),
                                float("-inf"))
        n = lg.numel()
        timed(f"softmax_{name}", lambda: K.softmax(masked), 4 * n, "pre-masked logits")
        vis = 8 * 32 * L * (L + 1) // 2
        timed(f"causal_softmax_{name}", lambda: K.softmax(lg, causal=True), 2 * vis + 2 * n,
              "mask applied in the kernel; masked keys not read")
        timed(f"softmax_{name}_f32_out", lambda: K.softmax(masked, out_dtype=torch.float32),
              2 * n + 4 * n, "half_to_float (HF softmax(dtype=float32))")
        del masked
        # HF eager attention's tail (scale, [B, 1, L, L] additive mask with the
        # dtype's lowest value, softmax in fp32, cast back) as one launch; the
        # same chain as PyTorch CUDA ops for comparison
        hf = torch.zeros(8, 1, L, L, dtype=dt, device=dev).masked_fill(
            torch.triu(torch.ones(L, L, dtype=torch.bool, device=dev), 1), torch.finfo(dt).min)
        sc = 128 ** -0.5
        timed(f"masked_softmax_{name}", lambda: K.masked_softmax(lg, hf, sc), 4 * n + hf.numel() * 2,
              "HF eager attention tail in one launch: x*scale + mask, softmax, cast")
        timed(f"masked_softmax_{name}_torch_chain", lambda: torch.softmax(
            lg * sc + hf, -1, dtype=torch.float32).to(dt), 4 * n + hf.numel() * 2,
            "the same tail as 4 PyTorch CUDA ops (bytes: the fused op's)")
        del lg, hf
    if want("softmax_bf16_1024x128256", "softmax_f32_8192x32000"):
        for dt, R, V in ((torch.bfloat16, 1024, 128256), (torch.float32, 8192, 32000)):
            lv = (3.0 * torch.randn(R, V, generator=g, device=dev)).to(dt)
            esz = lv.element_size()
            timed(f"softmax_{'bf16' if dt == torch.bfloat16 else 'f32'}_{R}x{V}",
                  lambda: K.softmax(lv), 2 * esz * lv.numel(), "vocabulary-long rows")
            del lv

    # broadcast add / mul on the stack's activation shape: the residual add,
    # a [hidden] weight broadcast over the rows, a [T, 1] per-row scale
    TA = 131072
    xa = torch.randn(TA, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    ya = torch.randn(TA, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    wv = torch.randn(HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    cv = torch.randn(TA, 1, generator=g, device=dev).to(torch.bfloat16)
    n = xa.numel()
    timed(f"add_bf16_{TA}x{HIDDEN}", lambda: K.add(xa, ya), 3 * n * BF16)
    timed(f"mul_bf16_{TA}x{HIDDEN}_by_row_vector", lambda: K.mul(xa, wv), 2 * n * BF16,
          "[hidden] weight broadcast over the rows")
    timed(f"mul_bf16_{TA}x{HIDDEN}_by_column", lambda: K.mul(xa, cv), 2 * n * BF16,
          "[T, 1] per-row scale")
    del xa, ya, wv, cv
    # config 4: reductions
    xf = torch.randn(65536, 8192, generator=g, device=dev)
    n = xf.numel()
    timed("sum_lastdim_f32_65536x8192", lambda: K.sum_lastdim(xf), 4 * n + 4 * 65536)
    timed("mean_lastdim_f32_65536x8192", lambda: K.mean_lastdim(xf), 4 * n + 4 * 65536)
    timed("amax_lastdim_f32_65536x8192", lambda: K.amax_lastdim(xf), 4 * n + 4 * 65536)
    timed("sum_all_f32_65536x8192", lambda: K.sum_all(xf), 4 * n + 4)
    timed("mean_all_f32_65536x8192", lambda: K.mean_all(xf), 4 * n + 4)
    timed("amax_all_f32_65536x8192", lambda: K.amax_all(xf), 4 * n + 4)
    del xf
    xa = torch.randn(65536, 32000, generator=g, device=dev).to(torch.bfloat16)
    timed("argmax_lastdim_bf16_65536x32000", lambda: K.argmax_lastdim(xa),
          2 * xa.numel() + 8 * 65536)
    del xa
    xi = torch.randint(-1000, 1001, (65536, 8192), generator=g, device=dev, dtype=torch.int32)
    timed("sum_i32_i64_lastdim_65536x8192", lambda: K.sum_i32_i64(xi, False),
          4 * xi.numel() + 8 * 65536)
    timed("sum_i32_i64_all_65536x8192", lambda: K.sum_i32_i64(xi, True), 4 * xi.numel() + 8)
    del xi
    # backward kernels (training through the path): bytes = inputs read once
    # + outputs written once
    xb = torch.randn(65536, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    dyb = torch.randn(65536, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    wb = (1 + 0.1 * torch.randn(HIDDEN, generator=g, device=dev)).to(torch.bfloat16)
    timed("rms_norm_backward_bf16_65536x4096", lambda: K.rms_norm_backward(dyb, xb, wb, EPS),
          3 * xb.numel() * BF16 + 2 * HIDDEN * BF16, "x, dy in; dx, dw out")
    del xb, dyb
    gb = torch.randn(16384, INTER, generator=g, device=dev).to(torch.bfloat16)
    ub = torch.randn(16384, INTER, generator=g, device=dev).to(torch.bfloat16)
    db = torch.randn(16384, INTER, generator=g, device=dev).to(torch.bfloat16)
    timed("swiglu_backward_bf16_16384x14336", lambda: K.swiglu_backward(db, gb, ub),
          5 * gb.numel() * BF16, "dout, gate, up in; dgate, dup out")
    del gb, ub, db
    lg = (3.0 * torch.randn(8, 32, 2048, 2048, generator=g, device=dev)).to(torch.bfloat16)
    yb = K.softmax(lg, causal=True)
    dyb = torch.randn(8, 32, 2048, 2048, generator=g, device=dev).to(torch.bfloat16)
    timed("softmax_backward_bf16_8x32x2048x2048", lambda: K.softmax_backward(dyb, yb),
          3 * yb.numel() * BF16, "dy, y in; dx out")
    del lg, yb, dyb
    torch.cuda.empty_cache()
    return out


def chain_configs(dev, g, timed, T=8192):
    """The Llama decoder chain at 8192 tokens on one GPU: RMSNorm(4096, eps
    1e-5) -> RoPE (q [T,32,128], k [T,8,128], theta 1e4, positions 0..T-1) ->
    SwiGLU [T,14336] -> residual add, inputs ~ N(0,1), weight 1 + N(0,0.1).
    Timed as one step four ways: the four b200 launches replayed as a CUDA
    graph; the same launches eager; three launches (SwiGLU and the residual
    add in one kernel) as a graph; the HF formulas on PyTorch's CUDA kernels
    (what the reference's cuda route runs).  Bytes: 147,456 per token plus
    the cos/sin rows (512 per token).  Also the Qwen3 q/k-norm -> RoPE
    (rms_norm_rope) at the same token count, 20,480 B/token."""
    from torch_fl import kernels as K

    bf = torch.bfloat16

    def rn(*shape, scale=1.0, loc=0.0):
        return (loc + scale * torch.randn(*shape, generator=g, device=dev)).to(bf)

    x, y = rn(T, HIDDEN), rn(T, HIDDEN)
    w = rn(HIDDEN, scale=0.1, loc=1.0)
    q, k = rn(1, T, HQ, HEAD), rn(1, T, HKV, HEAD)
    gt, up = rn(T, INTER), rn(T, INTER)
    cos, sin = rope_tables(0, T, dev)
    n, h = torch.empty_like(x), torch.empty_like(x)
    qo, ko, a = torch.empty_like(q), torch.empty_like(k), torch.empty_like(gt)

    def rms():
        K.rms_norm(x, w, EPS, out=n)

    def rope():
        K.rope_qk(q, k, cos, sin, layout="bshd", q_out=qo, k_out=ko)

    def swi():
        K.swiglu(gt, up, out=a)

    def add():
        K.add(x, y, out=h)

    def chain4():
        rms(); rope(); swi(); add()   # noqa: E702

    def chain3():
        rms(); rope()                 # noqa: E702
        K.swiglu_residual(gt, up, x, y, act_out=a, h_out=h)

    chain_bytes = (BYTES["rms_norm"] + BYTES["rope_qk"] + BYTES["swiglu"] + BYTES["residual_add"]
                   + TABLE_BYTES_PER_TOKEN) * T
    tag = f"llama_chain_T{T}"
    from torch_fl import _abi

    pdl = _abi.set_pdl(False)
    g4n, g3n = capture_graph(chain4), capture_graph(chain3)
    _abi.set_pdl(True)
    g4, g3 = capture_graph(chain4), capture_graph(chain3)
    _abi.set_pdl(pdl)
    timed(f"{tag}_graph", g4.replay, chain_bytes,
          "RMSNorm, RoPE, SwiGLU, residual add: 4 b200 launches replayed as one CUDA graph "
          "(programmatic dependent launch)", flush=True, tokens=T, reps_=20)
    timed(f"{tag}_graph_no_pdl", g4n.replay, chain_bytes,
          "the same graph captured without programmatic dependent launch", flush=True,
          tokens=T, reps_=20)
    timed(f"{tag}_eager", chain4, chain_bytes, "the same 4 launches, eager", flush=True,
          tokens=T, reps_=20)
    timed(f"{tag}_fused_graph", g3.replay, chain_bytes,
          "RMSNorm, RoPE, SwiGLU+residual in one kernel: 3 launches as one CUDA graph "
          "(programmatic dependent launch)", flush=True, tokens=T, reps_=20)
    timed(f"{tag}_fused_graph_no_pdl", g3n.replay, chain_bytes,
          "the same 3-launch graph without programmatic dependent launch", flush=True,
          tokens=T, reps_=20)
    del g4, g3, g4n, g3n

    def torch_chain():
        hf = x.to(torch.float32)
        hf = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + EPS)
        nn = w * hf.to(bf)
        qt, kt = q.transpose(1, 2), k.transpose(1, 2)
        c, s_ = cos[None, None], sin[None, None]

        def rot(t):
            return torch.cat((-t[..., HEAD // 2:], t[..., :HEAD // 2]), dim=-1)

        qe = (qt * c) + (rot(qt) * s_)
        ke = (kt * c) + (rot(kt) * s_)
        aa = torch.nn.functional.silu(gt) * up
        return nn, qe, ke, aa, x + y

    timed(f"{tag}_torch_eager", torch_chain, chain_bytes,
          "HF formulas on PyTorch CUDA eager kernels (the reference's cuda route)", flush=True,
          tokens=T, reps_=10)
    # the chain's kernels one at a time at this size
    timed(f"rms_norm_bf16_{T}x{HIDDEN}", rms, BYTES["rms_norm"] * T, flush=True, reps_=20)
    timed(f"rope_qk_bf16_T{T}", rope, (BYTES["rope_qk"] + TABLE_BYTES_PER_TOKEN) * T, flush=True,
          reps_=20)
    timed(f"swiglu_bf16_{T}x{INTER}", swi, BYTES["swiglu"] * T, flush=True, reps_=20)
    timed(f"add_bf16_{T}x{HIDDEN}", add, BYTES["residual_add"] * T, flush=True, reps_=20)
    del gt, up, a, x, y, n, h
    # Qwen3 q_norm / k_norm (per-head RMSNorm over 128, eps 1e-6, [128] weights)
    # then RoPE, one launch; bytes: q, k read and written + the table rows
    wq, wk = rn(HEAD, scale=0.1, loc=1.0), rn(HEAD, scale=0.1, loc=1.0)
    nr_bytes = (BYTES["rope_qk"] + TABLE_BYTES_PER_TOKEN) * T
    timed(f"rms_norm_rope_bf16_T{T}", lambda: K.rope_qk(
        q, k, cos, sin, layout="bshd", q_weight=wq, k_weight=wk, eps=1e-6, q_out=qo, k_out=ko),
        nr_bytes, "Qwen3-8B shapes: q [T,32,128], k [T,8,128], [128] norm weights", flush=True,
        tokens=T, reps_=20)
    TL = 131072
    q2, k2 = rn(1, TL, HQ, HEAD), rn(1, TL, HKV, HEAD)
    c2, s2 = rope_tables(0, TL, dev)
    timed(f"rms_norm_rope_bf16_T{TL}", lambda: K.rope_qk(
        q2, k2, c2, s2, layout="bshd", q_weight=wq, k_weight=wk, eps=1e-6, inplace=True),
        (BYTES["rope_qk"] + TABLE_BYTES_PER_TOKEN) * TL, "in place, inputs larger than L2",
        tokens=TL)
    del q2, k2, c2, s2, q, k, qo, ko


def stack_bytes(stack):
    """Algorithmic HBM bytes of one step on this rank."""
    T, L = stack.T, stack.L
    if stack.fuse:
        per = BYTES["rope_qk"] + BYTES["swiglu"]
        return T * (L * per + BYTES["rms_norm"] + (L - 1) * 4 * HIDDEN * BF16 + BYTES["residual_add"])
    return T * L * BYTES_PER_TOKEN_LAYER


# Small cases for ncu captures: each input larger than L2 (126 MB) and a few
# GB on the device at most; one launch of the op (after one warm-up launch).
PROFILE_CASES = {
    "stack": "2 layers of the stack on 16384 tokens (RMSNorm, RoPE, SwiGLU, add+RMSNorm, "
             "RoPE, SwiGLU+residual); warm-up step first",
    "softmax": "softmax bf16 [2, 32, 2048, 2048]",
    "causal_softmax": "causal softmax bf16 [2, 32, 2048, 2048]",
    "softmax_f16": "softmax f16 [1, 32, 4096, 4096]",
    "argmax": "argmax bf16 [8192, 32000]",
    "sum_all": "full sum f32 [16384, 8192]",
    "rms_norm_backward": "RMSNorm backward bf16 [16384, 4096] (dx and dw)",
    "swiglu_backward": "SwiGLU backward bf16 [4096, 14336]",
    "softmax_backward": "softmax backward bf16 [2, 32, 2048, 2048]",
    "masked_softmax": "scaled masked softmax bf16 [2, 32, 2048, 2048], HF mask [2, 1, 2048, 2048]",
    "softmax_long": "softmax bf16 [512, 128256] (a vocabulary of logits per row)",
    "elementwise": "add bf16 [32768, 4096] + [32768, 4096]; mul by a [4096] row vector; "
                   "mul by a [32768, 1] column",
    "causal_softmax_f16_4096": "causal softmax f16 [1, 32, 4096, 4096] (mask applied in the "
                               "kernel)",
    "masked_softmax_f16_4096": "scaled masked softmax f16 [1, 32, 4096, 4096], HF mask "
                               "[1, 1, 4096, 4096]",
    "chain_8192": "the 8192-token Llama chain: RMSNorm [8192, 4096], RoPE q [8192, 32, 128] / "
                  "k [8192, 8, 128], SwiGLU [8192, 14336], residual add [8192, 4096]; then "
                  "Qwen3 q/k-norm -> RoPE on the same q, k",
}


def profile_case(name):
    from torch_fl import kernels as K

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(11)
    if name == "stack":
        st = Stack(16384, 2, 0, dev, "fused", True)
        fn = lambda: st.run(st.x0)  # noqa: E731
    elif name in ("softmax", "causal_softmax"):
        x = (3.0 * torch.randn(2, 32, 2048, 2048, generator=g, device=dev)).to(torch.bfloat16)
        fn = lambda: K.softmax(x, causal=name == "causal_softmax")  # noqa: E731
    elif name == "softmax_f16":
        x = (3.0 * torch.randn(1, 32, 4096, 4096, generator=g, device=dev)).to(torch.float16)
        fn = lambda: K.softmax(x)  # noqa: E731
    elif name == "argmax":
        x = torch.randn(8192, 32000, generator=g, device=dev).to(torch.bfloat16)
        fn = lambda: K.argmax_lastdim(x)  # noqa: E731
    elif name == "sum_all":
        x = torch.randn(16384, 8192, generator=g, device=dev)
        fn = lambda: K.sum_all(x)  # noqa: E731
    elif name == "rms_norm_backward":
        x = torch.randn(16384, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
        dy = torch.randn(16384, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(HIDDEN, generator=g, device=dev)).to(torch.bfloat16)
        fn = lambda: K.rms_norm_backward(dy, x, w, EPS)  # noqa: E731
    elif name == "swiglu_backward":
        gt, up, d = (torch.randn(4096, INTER, generator=g, device=dev).to(torch.bfloat16)
                     for _ in range(3))
        fn = lambda: K.swiglu_backward(d, gt, up)  # noqa: E731
    elif name == "elementwise":
        a = torch.randn(32768, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
        b = torch.randn(32768, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
        wv = torch.randn(HIDDEN, generator=g, device=dev).to(torch.bfloat16)
        cv = torch.randn(32768, 1, generator=g, device=dev).to(torch.bfloat16)
        fn = lambda: (K.add(a, b), K.mul(a, wv), K.mul(a, cv))  # noqa: E731
    elif name == "softmax_long":
        x = (3.0 * torch.randn(512, 128256, generator=g, device=dev)).to(torch.bfloat16)
        fn = lambda: K.softmax(x)  # noqa: E731
    elif name == "chain_8192":
        T = 8192

        def rn(*shape, scale=1.0, loc=0.0):
            return (loc + scale * torch.randn(*shape, generator=g, device=dev)).to(torch.bfloat16)

        x, y, w = rn(T, HIDDEN), rn(T, HIDDEN), rn(HIDDEN, scale=0.1, loc=1.0)
        q, k = rn(1, T, HQ, HEAD), rn(1, T, HKV, HEAD)
        gt, up = rn(T, INTER), rn(T, INTER)
        wq, wk = rn(HEAD, scale=0.1, loc=1.0), rn(HEAD, scale=0.1, loc=1.0)
        cos, sin = rope_tables(0, T, dev)
        n, h, a = torch.empty_like(x), torch.empty_like(x), torch.empty_like(gt)
        qo, ko = torch.empty_like(q), torch.empty_like(k)
        fn = lambda: (K.rms_norm(x, w, EPS, out=n),  # noqa: E731
                      K.rope_qk(q, k, cos, sin, layout="bshd", q_out=qo, k_out=ko),
                      K.swiglu(gt, up, out=a), K.add(x, y, out=h),
                      K.rope_qk(q, k, cos, sin, layout="bshd", q_weight=wq, k_weight=wk,
                                eps=1e-6, q_out=qo, k_out=ko))
    elif name == "causal_softmax_f16_4096":
        x = (3.0 * torch.randn(1, 32, 4096, 4096, generator=g, device=dev)).to(torch.float16)
        fn = lambda: K.softmax(x, causal=True)  # noqa: E731
    elif name == "masked_softmax_f16_4096":
        x = (3.0 * torch.randn(1, 32, 4096, 4096, generator=g, device=dev)).to(torch.float16)
        m = torch.zeros(1, 1, 4096, 4096, dtype=torch.float16, device=dev).masked_fill(
            torch.triu(torch.ones(4096, 4096, dtype=torch.bool, device=dev), 1),
            torch.finfo(torch.float16).min)
        fn = lambda: K.masked_softmax(x, m, 128 ** -0.5)  # noqa: E731
    elif name == "masked_softmax":
        x = (3.0 * torch.randn(2, 32, 2048, 2048, generator=g, device=dev)).to(torch.bfloat16)
        m = torch.zeros(2, 1, 2048, 2048, dtype=torch.bfloat16, device=dev).masked_fill(
            torch.triu(torch.ones(2048, 2048, dtype=torch.bool, device=dev), 1),
            torch.finfo(torch.bfloat16).min)
        fn = lambda: K.masked_softmax(x, m, 128 ** -0.5)  # noqa: E731
    else:
        x = (3.0 * torch.randn(2, 32, 2048, 2048, generator=g, device=dev)).to(torch.bfloat16)
        y = K.softmax(x)
        dy = torch.randn(2, 32, 2048, 2048, generator=g, device=dev).to(torch.bfloat16)
        fn = lambda: K.softmax_backward(dy, y)  # noqa: E731
    fn()
    torch.cuda.synchronize()
    fn()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": name, "what": PROFILE_CASES[name]}))


def correctness_sample(stack, K, world, rank, dev):
    """Gather 4 rows of every rank's first-layer outputs to rank 0 and check
    them against the oracle (RoPE rows carry the global positions)."""
    rows = torch.tensor([0, 1, stack.T // 2, stack.T - 1], device=dev)
    n = K.rms_norm(stack.x0, stack.w[0], EPS, rounding=stack.rounding)
    stack._rope()
    a, h = K.swiglu_residual(stack.g, stack.u, stack.x0, stack.y, rounding=stack.rounding)
    parts = [stack.x0[rows], stack.y[rows], n[rows], stack.g[rows], stack.u[rows], a[rows], h[rows],
             stack.q[0, rows].reshape(4, -1), stack.qo[0, rows].reshape(4, -1),
             stack.cos[rows], stack.sin[rows]]
    flat = torch.cat([p.reshape(-1) for p in parts])
    if world > 1:
        import torch.distributed as dist

        out = torch.empty(world * flat.numel(), dtype=flat.dtype, device=dev)
        dist.all_gather_into_tensor(out, flat)
        gathered = out.view(world, -1)
    else:
        gathered = flat.view(1, -1)
    if rank != 0:
        return None
    import numpy as np

    from oracle import ops

    worst = 0
    table_ulp = 0
    sizes = [p.numel() for p in parts]
    w0 = stack.w[0].float().cpu().numpy()
    for r in range(world):
        vals = torch.split(gathered[r].float().cpu(), sizes)
        x, y, nn, g, u, a_, h_, q, qo, ct, st = [v.numpy().reshape(4, -1) for v in vals]
        # the rows' cos/sin are the rank's global positions r*T + {0, 1, T/2, T-1}
        pos = r * stack.T + np.array([0, 1, stack.T // 2, stack.T - 1])
        ct_o, st_o = ops.rope_tables(pos, HEAD, THETA, "bf16")
        table_ulp = max(table_ulp, int(max(ops.ulp_diff(ct, ct_o, "bf16").max(),
                                           ops.ulp_diff(st, st_o, "bf16").max())))
        checks = [
            (nn, ops.rms_norm_golden(x, w0, EPS, "bf16") if stack.rounding == "fused"
             else ops.rms_norm_chain(x, w0, EPS, "bf16")),
            (a_, ops.swiglu_golden(g, u, "bf16") if stack.rounding == "fused"
             else ops.swiglu_chain(g, u, "bf16")),
            (h_, ops.add_golden(x, y, 1.0, "bf16")),
        ]
        qref = (ops.rope_golden if stack.rounding == "fused" else ops.rope_chain)(
            q.reshape(4, HQ, HEAD), ct[:, None], st[:, None], "bf16").reshape(4, -1)
        checks.append((qo, qref))
        for got, ref in checks:
            worst = max(worst, int(ops.ulp_diff(got, ref, "bf16").max()))
    return {"max_ulp_vs_oracle": worst, "ranks_checked": world, "ok": worst <= 1 and table_ulp == 0,
            "rope_table_max_ulp_vs_oracle_tables": table_ulp}


if __name__ == "__main__":
    main()
