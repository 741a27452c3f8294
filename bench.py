"""Benchmark: spiking OCR seq2seq forward (teacher forcing) on B200.

Workload (the OCR seq2seq images/s configuration): per GPU a batch of 256
synthetic text-line images [1, 64, 1024] (U(0, 0.2) background plus 5-40
black rectangles of side 8-20 px, seeded), 16x16 patch embedding to D=384
(256 tokens), 8 spiking encoder + 4 spiking decoder layers (H=8, MLP 1536),
T=4, target sequences of 64 uniformly random byte tokens (vocab 256) with a
causal decoder mask, random-init weights rounded to bf16.  A step is one
forward pass over the batch.  Weak scaling: every rank runs its own batch,
no collective on the data path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the CPU oracle (the PyTorch restatement of the
reference modules, oracle/) on the host cores on a bounded sample of the same
workload; under torchrun only rank 0 runs it.

One JSON line on rank 0: the metric, the device-timed value, the end-to-end
value through host buffers (e2e), the roofline of the dominant kernel, one
roofline line per kernel family (the fused GEMM and attention launches of the
forward, the LIF scan alone), the three kernel families alone at their
benchmark configurations, the CPU baseline, the SM clocks sampled during the
timed region and the number of library kernel launches.  The timed region
only counts launches; per-kernel device times come from further steps with an
event pair around every launch.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "ocr_seq2seq_images_per_sec"
UNIT = "images/s"
ARCH = dict(patch_size=16, d_model=384, n_heads=8, ff_dim=1536, num_encoder_layers=8, num_decoder_layers=4,
            tgt_vocab_size=256, n_steps=4, image_encoder="patch")
IMG = (1, 64, 1024)
SEQ = 64


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="forward", choices=["forward", "train", "decode"],
                    help="forward: the OCR seq2seq forward (default); train: one DDP training step per step; "
                         "decode: batched greedy decoding of 64 tokens per image")
    ap.add_argument("--batch", type=int, default=None, help="images per GPU (forward 256, train 64, decode 64)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="run the timed steps eagerly (forward: instead of replaying a CUDA graph of the "
                         "forward; train: the one-GPU step)")
    ap.add_argument("--bucket-elems", type=int, default=4 << 20,
                    help="train, N > 1: gradient elements per all-reduce bucket")
    ap.add_argument("--surrogate", default="arctan", choices=["arctan", "superspike"],
                    help="train: LIF surrogate gradient (arctan alpha 2, the training benchmark's; superspike k 4, "
                         "the reference trainer's)")
    ap.add_argument("--no-kernel-configs", action="store_true",
                    help="forward: skip the standalone LIF / Linear-LN-LIF / attention timings")
    return ap.parse_args()


def synthetic_lines(B, seed, H=64, W=1024):
    g = torch.Generator().manual_seed(seed)
    img = torch.rand(B, 1, H, W, generator=g) * 0.2
    for b in range(B):
        n = int(torch.randint(5, 41, (1,), generator=g))
        hs = torch.randint(8, 21, (n, 2), generator=g)
        for i in range(n):
            h, w = int(hs[i, 0]), int(hs[i, 1])
            y = int(torch.randint(0, H - h + 1, (1,), generator=g))
            x = int(torch.randint(0, W - w + 1, (1,), generator=g))
            img[b, 0, y:y + h, x:x + w] = 0.0
    return img


def make_inputs(B, seed):
    src = synthetic_lines(B, seed)
    tgt = torch.randint(0, ARCH["tgt_vocab_size"], (B, SEQ), generator=torch.Generator().manual_seed(seed + 7))
    mask = torch.tril(torch.ones(SEQ, SEQ)).expand(B, 1, SEQ, SEQ).contiguous()
    return src, tgt, mask


def round_weights_bf16(model):
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, (torch.nn.Linear, torch.nn.Conv2d)):
                m.weight.copy_(m.weight.to(torch.bfloat16).float())


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def shard_seed(rank, i):
    """Seed of input set i on a rank: every rank draws its own images."""
    return 1000 * rank + i


def max_over_ranks(x, device):
    """The largest value of x over all ranks (one all-reduce of a scalar);
    x itself when no process group is running."""
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms.

    Start it before the warm-up steps (nvidia-smi takes a few hundred ms to
    print its first line) and bracket the timed region with begin() and
    end(): summary() keeps only the samples taken inside that window."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index, interval_ms=100):
        self.index = index
        self.interval_ms = interval_ms
        self.samples = []  # (host monotonic time, fields)
        self.proc = None
        self.t0 = None
        self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", str(self.interval_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def begin(self):
        self.t0 = time.monotonic()

    def end(self):
        self.t1 = time.monotonic()

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.proc = None

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.stop()
        return False

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append((time.monotonic(), parts))

    def window(self):
        """Samples inside [begin, end]; all of them when no window was marked."""
        lo = self.t0 if self.t0 is not None else float("-inf")
        hi = self.t1 if self.t1 is not None else float("inf")
        return [s for t, s in self.samples if lo <= t <= hi]

    def summary(self):
        samples = self.window()
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(s[0]) for s in samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in samples if s[1].replace(".", "").isdigit()]
        pw = [float(s[2]) for s in samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in samples for i in range(4) if s[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_median": statistics.median(pw) if pw else None,
                "reasons": reasons, "samples": len(samples), "interval_ms": self.interval_ms}


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum, one ncu capture of
# the same launch shape) of the kernels that can be the dominant one of the 256-image
# forward
NCU_TRAFFIC = {
    "linear_ln_lif K=384 N=384 rows=262144": 358.5e6,
    "linear_ln_lif K=384 N=384 rows=262144 +residual": 558.5e6,
    "linear_ln_lif K=384 N=1536 rows=262144": 950.6e6,
    "linear_ln_lif K=1536 N=384 rows=262144 +residual": 1212.4e6,
    "linear_ln_lif K=512 N=384 rows=65536": 211.3e6,
    "ssa Nq=256 Nk=256": 774.4e6,
    "ssa Nq=64 Nk=256": 493.4e6,
    "ssa Nq=64 Nk=64": 173.4e6,
}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def cpu_threads():
    """Use every host thread for the CPU legs (the cpu_baseline sample and the
    reference arm run the same way); returns the count."""
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def peak_for(bound, peaks, peak_src, clocks):
    """Roofline denominator: measured HBM copy bandwidth, or the bf16 dense
    GEMM peak in the regime the sampled clocks show (burst when the median SM
    clock under load stayed within 5% of its maximum, else sustained)."""
    if bound == "hbm":
        return peaks["hbm_gbs"], "HBM copy (%s)" % peak_src
    sm = (clocks or {}).get("sm_mhz")
    mx = (clocks or {}).get("sm_max_mhz") or peaks.get("sm_max_mhz")
    if sm is not None and mx and sm >= 0.95 * mx:
        return peaks["bf16_tflops"], ("bf16 dense, burst (%s): median SM clock %.0f of %.0f MHz in the timed region"
                                      % (peak_src, sm, mx))
    return (peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]),
            "bf16 dense, sustained (%s): median SM clock %s MHz in the timed region" % (peak_src, sm))


def roofline_entry(tag, rec, bound, peaks, peak_src, clocks):
    """achieved / peak of one launch kind from its recorded device time.

    ``bound`` None picks the binding roofline: the one whose minimum time for
    the launch's algorithmic work is longer (the fused GEMMs at K = N = 384
    move more bytes per FLOP than the bf16 ridge point and are HBM-bound).
    Both fractions are reported."""
    per_launch_s = rec["ms"] / rec["launches"] / 1000.0
    flops = rec["flops"] / rec["launches"]
    nbytes = rec["bytes"] / rec["launches"]
    t_peak, t_kind = peak_for("tensor", peaks, peak_src, clocks)
    h_peak, h_kind = peak_for("hbm", peaks, peak_src, clocks)
    t_min_tensor = flops / (t_peak * 1e12)
    t_min_hbm = nbytes / (h_peak * 1e9)
    if bound is None:
        bound = "tensor" if t_min_tensor >= t_min_hbm else "hbm"
    if bound == "tensor":
        achieved, unit, peak, kind = flops / per_launch_s / 1e12, "TFLOP/s", t_peak, t_kind
    else:
        achieved, unit, peak, kind = nbytes / per_launch_s / 1e9, "GB/s", h_peak, h_kind
    e = {"kernel": tag, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
         "peak_kind": kind, "ms_per_launch": per_launch_s * 1000.0, "launches_timed": rec["launches"],
         "algorithmic_bytes": nbytes, "algorithmic_flops": flops}
    if flops > 0 and nbytes > 0:
        e["frac_tensor"] = t_min_tensor / per_launch_s
        e["frac_hbm"] = t_min_hbm / per_launch_s
    return e


def config_kernels(dev, peaks, peak_src):
    """The three kernel families alone at their benchmark configurations,
    timed with CUDA events on the launching stream (each call after 3 warm-up
    calls, inputs rotated over copies whose total exceeds the 126 MB L2):

    * LIF scan at the MLP-expand shape of 64 images, [4, 64*256*1536] fp32
      N(0.5, 1), tau = 2 neuron: forward to packed-bit spikes and to bf16
      spikes, backward from packed-bit spikes;
    * fused Linear -> LayerNorm -> LIF, A [4*32*256, 384] Bernoulli(0.15) bf16,
      W [1536, 384] bf16, bf16 spikes;
    * attention core + LIF on [4, 32, 8, 256, 48] Bernoulli(0.15) spikes,
      plain ((Q K^T) V * 0.125) and XNOR forms, and the causal form at N = 64.

    Each measurement replays a CUDA graph of the calls.  Kernels timed alone:
    the bf16 peak is the burst figure."""
    from spikingtransformer_b200 import ops
    burst = {"sm_mhz": 1.0, "sm_max_mhz": 1.0}
    out = {}

    def timed(fn, reps):
        # the calls are captured once in a CUDA graph and replayed, so the
        # host's per-call overhead does not leave the GPU idle between them
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(reps):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / reps

    def add(name, bound, ms, nbytes=0.0, flops=0.0, note=None):
        rec = {"ms": ms, "launches": 1, "bytes": nbytes, "flops": flops}
        e = roofline_entry(name, rec, bound, peaks, peak_src, burst)
        if note:
            e["note"] = note
        out[name] = e

    g = torch.Generator(device=dev).manual_seed(0)
    # ---- LIF scan
    T, M = 4, 64 * 256 * 1536
    x = torch.randn(T, M, generator=g, device=dev).add_(0.5)
    ms = timed(lambda i: ops.lif_fwd(x, 0.5, 1.0, 0.0, in_gain=0.5, spike_dtype="bits"), 10)
    add("lif_fwd [4, 25165824] f32 -> packed-bit spikes", "hbm", ms, T * M * 4 + T * M / 8 + 4 * M)
    ms = timed(lambda i: ops.lif_fwd(x, 0.5, 1.0, 0.0, in_gain=0.5, spike_dtype=torch.bfloat16), 10)
    add("lif_fwd [4, 25165824] f32 -> bf16 spikes", "hbm", ms, T * M * 6 + 4 * M)
    sb, _ = ops.lif_fwd(x, 0.5, 1.0, 0.0, in_gain=0.5, spike_dtype="bits", want_v_final=False)
    gs = torch.randn(T, M, generator=g, device=dev)
    ms = timed(lambda i: ops.lif_bwd(gs, None, x, sb, 0.5, 1.0, 0.0, in_gain=0.5, spikes_packed=True), 10)
    add("lif_bwd [4, 25165824] f32, packed-bit spikes", "hbm", ms, T * M * 12 + T * M / 8,
        note="bytes: g_spikes, x and grad_x fp32 plus the packed spikes; the reference also writes and re-reads "
             "a [T, N] fp32 membrane history")
    del x, gs, sb
    # ---- fused Linear -> LayerNorm -> LIF
    R, K, N = 32 * 256, 384, 1536
    As = [(torch.rand(T * R, K, generator=g, device=dev) < 0.15).to(torch.bfloat16) for _ in range(6)]
    W = ((torch.rand(N, K, generator=g, device=dev) * 2 - 1) / math.sqrt(K)).to(torch.bfloat16)
    bias = (torch.rand(N, generator=g, device=dev) * 2 - 1) * 0.01
    ones, zeros = torch.ones(N, device=dev), torch.zeros(N, device=dev)
    ms = timed(lambda i: ops.linear_ln_lif(As[i % 6], W, bias, ones, zeros, 1e-5, 0.5, 1.0, 0.0, T, in_gain=0.5), 20)
    add("linear_ln_lif [32768, 384] x [384, 1536] -> bf16 spikes", None, ms,
        nbytes=(T * R * K + N * K) * 2 + T * R * N * 2, flops=2.0 * T * R * K * N)
    del As
    # ---- attention core + LIF
    for Ns, causal, nsets in ((256, False, 3), (64, True, 8)):
        B, H, dh = 32, 8, 48
        sets = [tuple((torch.rand(T * B, Ns, H * dh, generator=g, device=dev) < 0.15).to(torch.bfloat16)
                      for _ in range(3)) for _ in range(nsets)]
        nbytes = 4.0 * T * B * Ns * H * dh * 2  # q, k, v in, spikes out (bf16)
        dense = 4.0 * T * B * H * Ns * Ns * dh
        for variant, scale, vname in ((0, 0.125, "plain"), (1, (1.0 / dh) ** 0.5, "xnor")):
            ms = timed(lambda i: ops.ssa(*sets[i % nsets], T, B, H, variant, scale, 0.5, 0.5, 0.0, in_gain=0.5,
                                         causal=causal), 20)
            name = "ssa %s [4, 32, 8, %d, 48]%s" % (vname, Ns, " causal" if causal else "")
            add(name, "hbm", ms, nbytes=nbytes, flops=dense,
                note="%.1f dense-equivalent TFLOP/s (QK^T and SV counted dense)" % (dense / (ms / 1000.0) / 1e12))
        del sets
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def cpu_oracle_rate(target_s=12.0, max_batch=64):
    """Images/s of the CPU oracle forward on a bounded sample (all host threads)."""
    from oracle import modules as om
    cpu_threads()
    torch.manual_seed(0)
    m = om.Seq2Seq(**ARCH).eval()
    round_weights_bf16(m)
    B = 1
    with torch.no_grad():
        src, tgt, mask = make_inputs(B, 1234)
        t0 = time.perf_counter()
        m(src, tgt, look_ahead_mask=mask)
        per_img = time.perf_counter() - t0
        B = int(max(1, min(max_batch, target_s / max(per_img, 1e-3))))
        src, tgt, mask = make_inputs(B, 4321)
        t0 = time.perf_counter()
        m(src, tgt, look_ahead_mask=mask)
        dt = time.perf_counter() - t0
    return B / dt, B, dt


def run_reference(args, ws, rank):
    """--impl reference: the CPU oracle timed on the host cores."""
    if rank != 0:
        return
    from oracle import modules as om
    cpu_threads()
    torch.manual_seed(0)
    m = om.Seq2Seq(**ARCH).eval()
    round_weights_bf16(m)
    with torch.no_grad():
        src, tgt, mask = make_inputs(1, 99)
        t0 = time.perf_counter()
        m(src, tgt, look_ahead_mask=mask)
        per = time.perf_counter() - t0
        # bounded sample per step: the whole run stays within a few minutes
        budget = 150.0 / max(1, args.steps + args.warmup)
        B = int(max(1, min(16, budget / max(per, 1e-3))))
        src, tgt, mask = make_inputs(B, 100)
        for _ in range(args.warmup):
            m(src, tgt, look_ahead_mask=mask)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            m(src, tgt, look_ahead_mask=mask)
        dt = time.perf_counter() - t0
    rate = B * args.steps / dt
    cores = torch.get_num_threads()
    sample = "%d images [1,64,1024] per step, full 8+4-layer forward (PyTorch eager oracle, fp32)" % B
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * dt / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "ocr_seq2seq_forward", "per_step_images": B, "seq_len": SEQ, "image": list(IMG),
                   "T": 4, "d_model": 384, "layers": "8+4", "parallelism": "cpu"},
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_train(args, ws, rank, local):
    """--workload train: forward + backward + AdamW step of the same model, one
    process per GPU, gradients all-reduced by DDP over NCCL (bf16 autocast as
    the reference trains under fp16 autocast, train_spikeformer.py:545-555;
    loss = mean over T of CrossEntropyLoss(ignore_index=0, label_smoothing=0.1)
    of each step's logits, train_spikeformer.py:269,309-323, fused with the
    token accuracy).  The surrogate is the training benchmark's arctan with
    alpha = 2, which differs from the reference trainer's SuperSpike with
    k = 4 (Lif.py:280-282); --surrogate superspike selects that one.  Each step generates its
    batch on the device (images and byte targets from a per-rank, per-step
    seed), so no host data path enters the step."""
    import datetime
    import torch.distributed as dist
    from spikingtransformer_b200 import _lib, ops
    from spikingtransformer_b200.Seq2Seq import Seq2Seq
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    _lib.load()
    torch.manual_seed(0)  # same initial weights on every rank
    model = Seq2Seq(**ARCH)
    round_weights_bf16(model)
    if args.surrogate == "arctan":
        model.set_surrogate("arctan", 2.0)
    model = model.to(dev).train()
    # The forward, backward and optimizer step are captured once into a CUDA
    # graph (the host would otherwise spend longer enqueueing the step's ~2,000
    # launches than the GPU spends running them); each step generates its batch
    # into the graph's static input buffers and replays the graph.  With N > 1
    # every parameter's gradient is a view into one flat fp32 buffer whose
    # buckets are cast to bf16 and all-reduced over NCCL on a side stream as
    # the backward completes them (BucketedGradReducer), so the transfers
    # overlap the rest of the backward inside the graph.  --no-graph runs the
    # step eagerly (DDP with its bf16 compression hook for N > 1).
    use_graph = not args.no_graph
    net = model
    reducer = None
    if ws > 1 and not use_graph:
        from torch.distributed.algorithms.ddp_comm_hooks import default_hooks
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local], bucket_cap_mb=25,
                                                        gradient_as_bucket_view=True)
        net.register_comm_hook(None, default_hooks.bf16_compress_hook)
    if ws > 1 and use_graph:
        from spikingtransformer_b200.dp import BucketedGradReducer
        reducer = BucketedGradReducer(model.parameters(), bucket_elems=args.bucket_elems)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True, capturable=use_graph)
    B = args.batch or 64
    mask = torch.tril(torch.ones(SEQ, SEQ, device=dev)).expand(B, 1, SEQ, SEQ)

    def gen(i):
        return ops.synth_text_lines(B, 1_000_000 + shard_seed(rank, i), H=IMG[1], W=IMG[2], L=SEQ + 1,
                                    V=ARCH["tgt_vocab_size"], device=dev)

    def zero_grads():
        if reducer is not None:
            reducer.begin()  # the gradients stay views into its flat buffer
        else:
            opt.zero_grad(set_to_none=True)

    def train_step(src, labels):
        tgt_in, tgt_out = labels[:, :-1], labels[:, 1:]
        with torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=not use_graph):
            logits, _ = net(src, tgt_in, look_ahead_mask=mask)
        loss, acc, _ = ops.ce_over_t(logits, tgt_out, ignore_index=0, label_smoothing=0.1)
        loss.backward()
        if reducer is not None:
            reducer.finish()
        opt.step()
        return loss, acc

    graph_launches = None
    graphs = {}  # released before the process group (a graph that holds NCCL calls must go first)
    if use_graph:
        static_src, static_labels = gen(0)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for i in range(args.warmup):
                src, labels = gen(i)
                static_src.copy_(src)
                static_labels.copy_(labels)
                zero_grads()
                train_step(static_src, static_labels)
        torch.cuda.current_stream(dev).wait_stream(side)
        graphs["train"] = torch.cuda.CUDAGraph()
        if reducer is None:
            opt.zero_grad(set_to_none=True)
        with _lib.LaunchCounter() as counter, torch.cuda.graph(graphs["train"]):
            if reducer is not None:
                reducer.begin()
            g_loss, g_acc = train_step(static_src, static_labels)
        graph_launches = counter.total()

        def step(i):
            src, labels = gen(i)
            static_src.copy_(src)
            static_labels.copy_(labels)
            graphs["train"].replay()
            return g_loss, g_acc
    else:
        def step(i):
            src, labels = gen(i)
            zero_grads()
            return train_step(src, labels)

        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk, _lib.LaunchRecorder() as rec:
        # nvidia-smi prints its first sample a few hundred ms after it starts
        time.sleep(0.5)
        clk.begin()
        e0.record()
        for i in range(args.steps):
            loss, acc = step(args.warmup + i)
        e1.record()
        torch.cuda.synchronize()
        clk.end()
    if ws > 1:
        dist.barrier()
    ms = max_over_ranks(e0.elapsed_time(e1), dev)
    last, last_acc = float(loss.item()), float(acc.item())
    kernels = rec.summary()
    if rank == 0:
        print(json.dumps({
            "metric": "ocr_seq2seq_train_images_per_sec", "value": ws * B * args.steps / (ms / 1000.0),
            "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic, generated on the device each step",
            "config": {"workload": "ocr_seq2seq_train_step", "global_batch": ws * B, "per_gpu_batch": B,
                       "seq_len": SEQ, "image": list(IMG), "T": 4, "layers": "8 enc + 4 dec",
                       "optimizer": "AdamW lr 1e-4",
                       "surrogate": "arctan alpha 2" if args.surrogate == "arctan" else "superspike k 4",
                       "loss": "mean over T of CE(ignore_index=0, label_smoothing=0.1), fused with token accuracy",
                       "parallelism": ("dp%d (bf16 gradient buckets all-reduced over NCCL on a side stream as the "
                                       "backward completes them, inside the CUDA graph)" % ws if reducer is not None
                                       else "ddp%d (NCCL all-reduce of bf16-compressed gradient buckets)" % ws
                                       if ws > 1 else "single GPU")},
            "loss": last, "token_accuracy": last_acc, "clocks": clk.summary(),
            "cuda_graph": use_graph, "graph_launches_per_step": graph_launches,
            "gpu_launches": sum(v["launches"] for v in kernels.values()) + (graph_launches or 0) * args.steps,
            "kernels": {k: {"launches": v["launches"], "ms_per_step": v["ms"] / args.steps}
                        for k, v in sorted(kernels.items(), key=lambda kv: -kv[1]["ms"])},
        }), flush=True)
    graphs.clear()
    step = None
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_decode(args, ws, rank, local):
    """--workload decode: greedy decoding (``Seq2Seq.py:136-162``) of a batch of
    images per GPU, 64 tokens each (no eos, so every image runs all steps),
    through ``greedy_decode_batch``; beside it the per-image ``greedy_decode``
    loop of the reference's API on a few images of the same batch."""
    import datetime
    import torch.distributed as dist
    from spikingtransformer_b200 import _lib
    from spikingtransformer_b200.Seq2Seq import Seq2Seq
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    _lib.load()
    torch.manual_seed(0)
    model = Seq2Seq(**ARCH)
    round_weights_bf16(model)
    model = model.to(dev).eval()
    B = args.batch or 64
    max_len = SEQ + 1
    src, _, _ = make_inputs(B, shard_seed(rank, 0))
    src = src.to(dev)

    def batch_decode():
        return model.greedy_decode_batch(src, max_len=max_len, start_symbol=1, eos_idx=-1, pad_idx=0, device=dev)

    for _ in range(max(1, args.warmup)):
        ys, _ = batch_decode()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    steps = max(1, args.steps // 4)
    with ClockSampler(local) as clk, _lib.LaunchRecorder() as rec:
        time.sleep(0.5)
        clk.begin()
        e0.record()
        for _ in range(steps):
            ys, _ = batch_decode()
        e1.record()
        torch.cuda.synchronize()
        clk.end()
    ms = max_over_ranks(e0.elapsed_time(e1), dev) / steps
    kernels = rec.summary()
    # the reference API: one image at a time
    n_single = 2
    model.greedy_decode(src[0], max_len=max_len, start_symbol=1, eos_idx=-1, pad_idx=0, device=dev)
    torch.cuda.synchronize()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record()
    for b in range(n_single):
        y1, _, _ = model.greedy_decode(src[b], max_len=max_len, start_symbol=1, eos_idx=-1, pad_idx=0, device=dev)
    s1.record()
    torch.cuda.synchronize()
    single_ms = s0.elapsed_time(s1) / n_single
    assert torch.equal(y1[0], ys[n_single - 1]), "batched and single-image decodes differ"
    if rank == 0:
        print(json.dumps({
            "metric": "ocr_greedy_decode_images_per_sec", "value": ws * B / (ms / 1000.0), "unit": UNIT,
            "n_gpus": ws, "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "ocr_greedy_decode", "per_gpu_batch": B, "tokens_per_image": max_len - 1,
                       "image": list(IMG), "T": 4, "layers": "8 enc + 4 dec",
                       "parallelism": "dp%d (batch-sharded, no collective)" % ws},
            "single_image_decode": {"ms_per_image": single_ms, "images_per_sec": 1000.0 / single_ms,
                                    "api": "greedy_decode, one image per call"},
            "clocks": clk.summary(), "gpu_launches": sum(v["launches"] for v in kernels.values()) // steps,
        }), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    ws, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    if args.workload == "train":
        run_train(args, ws, rank, local)
        return
    if args.workload == "decode":
        run_decode(args, ws, rank, local)
        return
    if args.batch is None:
        args.batch = 256
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import spikingtransformer_b200 as pkg
    from spikingtransformer_b200 import _lib, ops
    from spikingtransformer_b200.Seq2Seq import Seq2Seq
    from spikingtransformer_b200.streaming import stream_forward
    _lib.load()

    torch.manual_seed(0)
    model = Seq2Seq(**ARCH)
    round_weights_bf16(model)
    model = model.to(dev).eval()

    B = args.batch
    # four input sets (4 x 67 MB of images > 126 MB L2), rotated between steps
    sets = []
    for i in range(4):
        src, tgt, mask = make_inputs(B, shard_seed(rank, i))
        sets.append((src.to(dev), tgt.to(dev), mask.to(dev)))
    torch.cuda.synchronize()

    def eager_step(i):
        src, tgt, mask = sets[i % len(sets)]
        logits, _ = model(src, tgt, look_ahead_mask=mask)
        return logits

    # The timed steps replay a CUDA graph of the forward (the same kernels,
    # without the gaps between launches that eager enqueueing leaves): each
    # step copies its input set into the graph's static input buffers, then
    # replays.  The per-kernel pass and the end-to-end run below stay eager.
    graph, graph_launches = None, 0
    if not args.no_graph:
        static = [t.clone() for t in sets[0]]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.no_grad(), torch.cuda.stream(side):
            model(static[0], static[1], look_ahead_mask=static[2])  # tensor maps, caches, attributes
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), _lib.LaunchCounter() as gcount, torch.cuda.graph(graph):
            static_logits = model(static[0], static[1], look_ahead_mask=static[2])[0]
        graph_launches = gcount.total()

    def step(i):
        if graph is None:
            return eager_step(i)
        src, tgt, mask = sets[i % len(sets)]
        static[0].copy_(src)
        static[1].copy_(tgt)
        static[2].copy_(mask)
        graph.replay()
        return static_logits

    with torch.no_grad():
        clk = ClockSampler(local).start()
        try:
            for i in range(args.warmup):
                step(i)
            torch.cuda.synchronize()
            if ws > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            # the timed region: only launches counted (no events between kernels)
            with _lib.LaunchCounter() as counter:
                clk.begin()
                e0.record()
                for i in range(args.steps):
                    step(i)
                e1.record()
                torch.cuda.synchronize()
                clk.end()
        finally:
            clk.stop()
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1), dev)
        ops.device_error_check()
        clocks = clk.summary()
        # per-kernel device times in a separate pass (an event pair around every launch)
        n_rec = min(args.steps, 5)
        with _lib.LaunchRecorder() as rec:
            for i in range(n_rec):
                eager_step(i)
        kernels = rec.summary()

        # ---- end to end through the public API: pinned host inputs in, logits out
        e2e = None
        if not args.no_e2e:
            hsrc = [s[0].cpu().pin_memory() for s in sets]
            htgt = [s[1].cpu().pin_memory() for s in sets]
            hmask = [s[2].cpu().pin_memory() for s in sets]
            # logits [T, B, seq, vocab] fp32, two pinned buffers used in turn
            out_host = [torch.empty((4, B, SEQ, ARCH["tgt_vocab_size"]), dtype=torch.float32).pin_memory()
                        for _ in range(2)]
            h2d = hsrc[0].numel() * 4 + htgt[0].numel() * 8 + hmask[0].numel() * 4
            d2h = out_host[0].numel() * 4

            def fwd(src, tgt, mask):
                return model(src, tgt, look_ahead_mask=mask)[0]

            order = [j % 4 for j in range(args.steps)]
            stream_forward(fwd, [(hsrc[j], htgt[j], hmask[j]) for j in range(2)], [out_host[j] for j in range(2)])
            torch.cuda.synchronize()
            if ws > 1:
                dist.barrier()
            f0 = torch.cuda.Event(enable_timing=True)
            f1 = torch.cuda.Event(enable_timing=True)
            f0.record()
            # every step copies its own images, tokens and mask in and its logits out
            stream_forward(fwd, [(hsrc[j], htgt[j], hmask[j]) for j in order], [out_host[j % 2] for j in order])
            f1.record()
            torch.cuda.synchronize()
            ems = max_over_ranks(f0.elapsed_time(f1), dev)
            e2e = {"value": ws * B * args.steps / (ems / 1000.0), "unit": UNIT, "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h, "ms_per_step": ems / args.steps}

    launches = counter.total() + graph_launches * args.steps
    peaks, peak_src = measured_peaks()

    def bound_of(tag):
        # the attention kernels are memory-bound (score-free regrouping, FLOPs
        # counted dense-equivalent); for the fused GEMMs the binding roofline
        # of each shape is picked from its FLOPs and bytes
        return "hbm" if tag.startswith("ssa") or kernels[tag]["flops"] == 0 else None

    # dominant kernel = largest total device time per step
    dom_tag, dom = max(kernels.items(), key=lambda kv: kv[1]["ms"])
    roof = roofline_entry(dom_tag, dom, bound_of(dom_tag), peaks, peak_src, clocks)
    roof["traffic"] = NCU_TRAFFIC.get(dom_tag) if B == 256 else None
    roof["traffic_unit"] = "bytes per launch (ncu dram read + write)"
    # one line per kernel family: the fused GEMMs and the attention launches of the
    # forward (from the recorded pass), the LIF scan from its standalone timing
    by_family = {}
    for fam, pick in (("linear_ln_lif", lambda t: t.startswith("linear_ln_lif")), ("ssa", lambda t: t.startswith("ssa"))):
        tags = sorted((t for t in kernels if pick(t)), key=lambda t: -kernels[t]["ms"])
        by_family[fam] = [roofline_entry(t, kernels[t], bound_of(t), peaks, peak_src, clocks) for t in tags]
    cfg_kernels = None
    if rank == 0 and not args.no_kernel_configs:
        cfg_kernels = config_kernels(dev, peaks, peak_src)
        by_family["lif"] = [v for k, v in cfg_kernels.items() if k.startswith("lif")]

    if rank == 0:
        value = ws * B * args.steps / (ms / 1000.0)
        cpu = None
        if not args.no_cpu_baseline and ws == 1:
            rate, nb, dt = cpu_oracle_rate()
            cpu = {"value": rate, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                   "sample": "%d images [1,64,1024], one full 8+4-layer forward of the PyTorch eager oracle "
                             "(fp32), %.1f s" % (nb, dt)}
        breakdown = {k: {"launches": v["launches"] // n_rec, "ms_per_step": v["ms"] / n_rec,
                         "share": v["ms"] / max(1e-9, sum(x["ms"] for x in kernels.values()))}
                     for k, v in sorted(kernels.items(), key=lambda kv: -kv[1]["ms"])}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "ocr_seq2seq_forward", "global_batch": ws * B, "per_gpu_batch": B,
                       "seq_len": SEQ, "image": list(IMG), "T": 4, "d_model": 384, "heads": 8, "ff_dim": 1536,
                       "layers": "8 enc + 4 dec", "vocab": 256, "parallelism": "dp%d (batch-sharded, no collective)" % ws,
                       "l2": "inputs rotate over 4 sets of 67 MB images (> 126 MB L2); activations per step >> L2",
                       "timed_steps": ("CUDA graph replay of the forward; each step first copies its input set "
                                       "into the graph's input buffers") if graph is not None else "eager"},
            "e2e": e2e, "roofline": roof, "roofline_by_family": by_family, "cpu_baseline": cpu, "clocks": clocks,
            "cuda_graph": graph is not None,
            "gpu_launches": launches, "gpu_launches_per_step": launches // args.steps,
            "kernels": breakdown, "kernels_note": "per-kernel device times from %d further steps with an event pair "
                                                  "around every launch (not the timed region)" % n_rec,
            "kernel_configs": cfg_kernels,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
