"""Benchmark of the product-key memory (PKM) layer on B200: tokens/s of fwd + bwd + optimizer step.

    python bench.py [--gpus N --steps K --warmup W] [--impl cuda|reference] [--rows-per-half 4096]

Workload (BASELINE metric "PKM layer tokens/s (fwd+bwd+opt) at 16.8M rows"): one PKM layer with 4096 sub-keys
per half (16,777,216 value rows x 384, fp32 table, fp32 Adam moments), H=4 heads x knn=32 reads per token,
k_dim 256, d_model 384, no BatchNorm / swilu (the config-1 layer), 32,768 tokens per GPU per step, x ~ N(0, 1)
and upstream gradient ~ N(0, 1), seeded synthetic data. One step = forward under bf16 autocast (query
projection, sub-key scoring, selection, value bag), backward (value bag -> row store, selection -> scores ->
keys / query), value clipping, LazyRowAdam on the table + fused AdamW on the dense parameters. All through the
public API (smlm_b200.pkm.ProductKeyMemory, smlm_b200.sparse_values).

`value` is device-timed with the inputs resident (CUDA events on the launching stream, barrier + synchronize
around exactly K steps, max over ranks); on one GPU the step is captured once as a CUDA graph
(smlm_b200.graph_step.GraphedStep) and replayed, so the host does not limit it (the eager step is reported beside
it under `eager`). `e2e` repeats the K steps with each step's inputs copied from pinned
host memory and a scalar read back inside the timed region. `roofline` is the dominant kernel (the lazy Adam
step) against the measured HBM copy bandwidth. `cpu_baseline` times the reference's PyTorch CPU path (a
restatement under oracle/, the only oracle use in this file) on a bounded sample.

--impl reference times the reference's PyTorch path on the host cores instead (rank 0 only under torchrun).
With --gpus N > 1 (torchrun, one process per GPU, NCCL) the 16.8M-row table and its optimizer state are
row-sharded over the N GPUs and each GPU runs 32,768 tokens per step (weak scaling): the lookups, partial bags
and weight gradients cross NVLink through peer memory inside the owner kernels, the output gradients through an
NCCL all-gather, the replicated parameters' gradients through an NCCL all-reduce; the line's `exchange` key gives
the exchange calls' NVLink and HBM bytes against the measured peer-copy and HBM bandwidths.

The default run also measures the B-16M inference token loop (`inference`: prefill and greedy decode of the
B-16M model, per-token lookup latency). --case configs times BASELINE configs 1-4 as single layers (fwd / bwd /
opt separately; config 2 also with the forward reading a bf16 copy of the fp32 table, config 4 with its inputs from a
uniform + Zipf(1.1) token mix); --case model times BASELINE config 2 as stated, the B-1M model's training step;
--case scoring and --case inference run one part alone; --case engram times the Engram n-gram memory module;
--case host times the B-16M layer with its table in host RAM against the reference's own host-table path.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "sparse-memory-lm_b200"))
sys.path.insert(0, ROOT)

METRIC = "PKM layer tokens/s (fwd+bwd+opt) at 16.8M rows"
# DRAM bytes (read + write) of the fused row-sum + lazy Adam step per touched row, from the ncu capture of that
# kernel on a 1M-row layer; traffic scales with the touched rows.
ADAM_TRAFFIC_PER_ROW = 9575
# the same for the plain lazy Adam step over a written accumulator (ncu capture of lazy_adam_kernel, 1M rows)
ADAM_UNFUSED_TRAFFIC_PER_ROW = 10698
D_MODEL, HEADS, KNN, K_DIM = 384, 4, 32, 256
# peer copy bandwidth per direction per GPU measured over NVLink on this pool's B200s (nominal 900 GB/s)
NVLINK_PEER_GBS = 770.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--rows-per-half", type=int, default=4096, help="sub-keys per half (rows = this squared)")
    ap.add_argument("--tokens", type=int, default=32768, help="tokens per GPU per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-rows-per-half", type=int, default=1024)
    ap.add_argument("--cpu-tokens", type=int, default=4096)
    ap.add_argument("--case", choices=["layer", "scoring", "inference", "configs", "engram", "model", "host"],
                    default="layer",
                    help="scoring: only the fused sub-key scoring + selection of the workload's layer (a small "
                         "standalone case for profiler captures; prints its time per call); inference: only the "
                         "B-16M prefill / decode measurement; configs: BASELINE configs 1-4 as single layers "
                         "with fwd / bwd / opt timed separately (config 4 with a uniform + Zipf token mix); "
                         "model: BASELINE config 2, the B-1M model's training step; engram: the reference's "
                         "default Engram module (hash, one-lookup bags, backward, lazy Adam) per step; host: the "
                         "B-16M layer with its table in host RAM, this build against the reference's own host "
                         "path, per configuration (Adam, rowrms, rowrms + GACC, rowrms + HOT 5% + GACC)")
    ap.add_argument("--host-arm", choices=["both", "this_build", "reference"], default="both",
                    help="--case host: which implementations to time")
    ap.add_argument("--host-configs", default="adam,rowrms,rowrms+gacc,rowrms+hot5%+gacc",
                    help="--case host: comma-separated configurations to time")
    ap.add_argument("--model", choices=["b1m", "b16m"], default="b1m",
                    help="--case model: b1m = BASELINE config 2 (the B-1M step, one CUDA graph); b16m = the "
                         "reference's B-16M-sparse training step (12 layers, three memory layers sharing the "
                         "16.8M-row table, 32 x 1024 tokens), eager, beside the reference's own run of it")
    ap.add_argument("--micro-batch", type=int, default=0,
                    help="--case model --model b16m: sequences per forward / backward, gradients accumulated over "
                         "the step's 32 (0: all 32 at once; the reference's run used 4)")
    ap.add_argument("--no-inference", action="store_true", help="leave the inference measurement out of the line")
    ap.add_argument("--eager", action="store_true",
                    help="time the step as eager calls (default on one GPU: the step captured as one CUDA graph)")
    return ap.parse_args()


def run_scoring_case(args):
    """The fused tensor-core scoring + selection alone at the workload's shape (bf16 queries and keys), for
    profiler captures of score_topk_kernel / pk_pairs_kernel on a few hundred MB."""
    from smlm_b200 import kernels as K
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(5)
    n_keys, N = args.rows_per_half, args.tokens
    q = torch.randn(N, HEADS, K_DIM, device=dev, generator=gen).bfloat16()
    keys = (torch.randn(HEADS, 2, n_keys, K_DIM // 2, device=dev, generator=gen) * (K_DIM // 2) ** -0.5).bfloat16()
    for _ in range(args.warmup):
        K.score_select(q, keys, KNN)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        K.score_select(q, keys, KNN)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    print(json.dumps({"case": "scoring", "tokens": N, "rows_per_half": n_keys, "ms_per_call": round(ms, 4),
                      "flops_per_call": 2 * N * HEADS * 2 * n_keys * (K_DIM // 2)}), flush=True)


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------------------------- clocks
class Clocks:
    """nvidia-smi sampling of SM clocks / throttle reasons during a timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        try:
            rows = [ln.split(",") for ln in open(self.file.name).read().strip().splitlines() if ln.strip()]
            os.unlink(self.file.name)
        except OSError:
            rows = []
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows if len(r) >= 9 for n, v in zip(names, r[5:9]) if "Active" in v
                          and "Not" not in v})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


# ------------------------------------------------------------------------------------------------ layer
def build_layer(n_keys, device, world=1, capturable=False):
    from smlm_b200.pkm import ProductKeyMemory
    from smlm_b200.sparse_values import LazyRowAdam, OptimizerSet
    torch.manual_seed(0)
    group = torch.distributed.group.WORLD if world > 1 else None
    with torch.device(device):
        mem = ProductKeyMemory(D_MODEL, D_MODEL, n_keys=n_keys, heads=HEADS, knn=KNN, k_dim=K_DIM,
                               query_norm="none", swilu=False, value_grad="row_sparse", shard_group=group)
        # config-1 initialisation: query N(0, 0.02), bias 0, sub-keys N(0, 1/128), values N(0, 384^-0.5)
        with torch.no_grad():
            mem.query_proj.weight.normal_(0, 0.02)
            mem.keys.normal_(0, (K_DIM // 2) ** -0.5)
    if world > 1:
        from smlm_b200.sharded import broadcast_replicated
        broadcast_replicated(mem, group)
    table = mem.values.weight
    dense = [p for p in mem.parameters() if p is not table]
    opt = OptimizerSet(torch.optim.AdamW(dense, lr=1e-3, betas=(0.9, 0.98), weight_decay=0.0, fused=True,
                                         capturable=capturable),
                       LazyRowAdam([table], lr=1e-3, betas=(0.9, 0.98), eps=1e-8, capturable=capturable))
    return mem, opt


def train_step(mem, opt, x, g):
    from smlm_b200.sparse_values import clip_row_sparse
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = mem(x)
    out.backward(g)
    if mem.shard is not None:
        from smlm_b200.sharded import allreduce_replicated_grads
        allreduce_replicated_grads(mem, mem.shard_group)
    vnorm = clip_row_sparse([mem.values.weight], 1.0)
    torch.nn.utils.clip_grad_norm_([p for p in mem.parameters() if p.grad is not None], 1.0, foreach=True)
    opt.step()
    opt.zero_grad(set_to_none=True)
    return vnorm


def exchange_rooflines(per_kernel_ms, world, n, k, d, hbm_gbs, table_bytes=4):
    """Roofline of the row-sharded exchange calls of one rank and step (the owner kernels that read and write the
    other ranks' memory over NVLink), from their mean CUDA-event times `per_kernel_ms` (name -> ms); None on one
    GPU. n tokens per rank, k lookups per token (m = n k), d values per row; lookups spread evenly over the shards.
      xchg_forward      NVLink: this owner's buckets of the P-1 peers' lookups read (m / P entries of 12 B each),
                        a partial bag per peer token written (d x 4 B); HBM: this rank's lookups bucketed (read 8 B,
                        written 12 B each), this shard's ~m table rows, the dense local copy of the served lookups
                        (P m x 4 B cleared, m x 8 B written), the P partial slots summed into the output
      xchg_backward_gw  NVLink: the weight gradient of each remote in-shard lookup stored into its rank (4 B);
                        HBM: the all-gathered output gradients, this shard's ~m table rows, every rank's lookups
    Each call's target time is the slower of its NVLink bytes at NVLINK_PEER_GBS and its HBM bytes at hbm_gbs;
    frac = target / measured."""
    if world < 2:
        return None
    m = n * k
    calls = {
        "xchg_forward": ((world - 1) * (m // world) * 12 + (world - 1) * n * d * 4,
                         m * 20 + m * d * table_bytes + world * m * 4 + m * 8 + (world + 1) * n * d * 4),
        "xchg_backward_gw": ((world - 1) * m * 4 // world,
                             m * d * table_bytes + world * n * d * 4 + world * n * k * 4),
    }
    out = {}
    for name, (nv, hb) in calls.items():
        ms = per_kernel_ms.get(name)
        if not ms:
            continue
        t_nv, t_hbm = nv / (NVLINK_PEER_GBS * 1e9) * 1e3, hb / (hbm_gbs * 1e9) * 1e3
        nv_gbs, hb_gbs = nv / (ms / 1e3) / 1e9, hb / (ms / 1e3) / 1e9
        out[name] = {"ms": round(ms, 4), "nvlink_bytes": nv, "nvlink_GB/s": round(nv_gbs, 1),
                     "nvlink_frac": round(nv_gbs / NVLINK_PEER_GBS, 3), "hbm_bytes": hb, "hbm_GB/s": round(hb_gbs, 1),
                     "hbm_frac": round(hb_gbs / hbm_gbs, 3), "bound": "nvlink" if t_nv >= t_hbm else "hbm",
                     "target_ms": round(max(t_nv, t_hbm), 4), "frac": round(max(t_nv, t_hbm) / ms, 3)}
    return out


def timed_loop(fn, steps, world):
    """Device time (CUDA events around exactly `steps` calls, synchronised on both sides) and the host time the
    loop took to enqueue them (ms). Host time close to device time means the loop is host-bound."""
    barrier(world)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    t0 = time.perf_counter()
    for i in range(steps):
        fn(i)
    host = (time.perf_counter() - t0) * 1e3
    e.record()
    torch.cuda.synchronize()
    barrier(world)
    return s.elapsed_time(e), host


def run_cuda(args, world, rank, local):
    from smlm_b200 import _lib as L
    dev = torch.device("cuda", local)
    N, n_keys = args.tokens, args.rows_per_half
    # the step is captured as one CUDA graph (smlm_b200.graph_step), which takes the host out of the step (the
    # headline figures); on N > 1 GPUs the graph holds the peer exchange (device-side epochs) and the NCCL calls
    graphed = not args.eager
    mem, opt = build_layer(n_keys, dev, world, capturable=graphed)
    rows = mem.values.weight.shape[0]           # this GPU's rows (all of them on one GPU)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    n_batches = 4
    xs = [torch.randn(N, D_MODEL, device=dev, generator=gen) for _ in range(n_batches)]
    gs = [torch.randn(N, D_MODEL, device=dev, generator=gen) for _ in range(n_batches)]
    if graphed:
        # captured before any eager step: the warm-up steps run inside GraphedStep on its side stream (autograd
        # ties each parameter's gradient accumulation to the stream of its first backward, and the legacy
        # default stream cannot join a capture)
        from smlm_b200.graph_step import GraphedStep
        gstep = GraphedStep(lambda x, g: train_step(mem, opt, x, g), [xs[0], gs[0]], opt.opts,
                            warmup=args.warmup)
    else:
        for i in range(args.warmup):
            train_step(mem, opt, xs[i % n_batches], gs[i % n_batches])
    torch.cuda.synchronize()

    # unique rows per step (U) for the algorithmic byte counts: measured on untimed steps
    from smlm_b200.sparse_values import row_store
    st = row_store(mem.values.weight)
    uniq = []
    for i in range(2):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = mem(xs[i])
        out.backward(gs[i])
        if mem.shard is not None:
            from smlm_b200.sharded import allreduce_replicated_grads
            allreduce_replicated_grads(mem, mem.shard_group)
        uniq.append(st.touched_rows())
        opt.step()
        opt.zero_grad(set_to_none=True)
    U = sum(uniq) / len(uniq)

    eager_ms, eager_host_ms = timed_loop(lambda i: train_step(mem, opt, xs[i % n_batches], gs[i % n_batches]),
                                         args.steps, world)
    # per-kernel timings: the same number of further eager steps with CUDA events recorded around every library
    # call on the stream it launches on (kept out of the timed loops, whose host work they would add to)
    L.PROFILE = []
    timed_loop(lambda i: train_step(mem, opt, xs[i % n_batches], gs[i % n_batches]), args.steps, world)
    prof, L.PROFILE = L.PROFILE, None
    eager_ms = max_over_ranks(eager_ms, world)
    step_fn = lambda i, x, g: train_step(mem, opt, x, g)  # noqa: E731
    if graphed:
        step_fn = lambda i, x, g: gstep(x, g)  # noqa: E731
    with Clocks(local) as clocks:
        ms, host_ms = timed_loop(lambda i: step_fn(i, xs[i % n_batches], gs[i % n_batches]), args.steps, world)
    ms = max_over_ranks(ms, world)
    ms_step = ms / args.steps
    tokens_per_s = N * world / (ms_step / 1e3)
    per_kernel = {}
    launches = 0
    for name, s, e, nl in prof:
        per_kernel.setdefault(name, []).append(s.elapsed_time(e))
        launches += nl

    # end to end: every step's inputs copied from pinned host memory (on a copy stream, one step ahead, into two
    # alternating device buffers, so the copy of step i + 1 overlaps the compute of step i; step 0's copy is
    # inside the timed region too) and the step's clip norm read back to pinned host memory
    hx = [x.cpu().pin_memory() for x in xs]
    hg = [g.cpu().pin_memory() for g in gs]
    out_host = torch.empty(n_batches, dtype=torch.float32).pin_memory()
    copy_stream = torch.cuda.Stream(dev)
    bufs = [(torch.empty_like(xs[0]), torch.empty_like(gs[0])) for _ in range(2)]
    loaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def prefetch(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            if i >= 2:
                copy_stream.wait_event(consumed[b])          # step i - 2 is done with this buffer
            bufs[b][0].copy_(hx[i % n_batches], non_blocking=True)
            bufs[b][1].copy_(hg[i % n_batches], non_blocking=True)
            loaded[b].record(copy_stream)

    def e2e_step(i):
        if i == 0:
            copy_stream.wait_stream(torch.cuda.current_stream(dev))  # after the timed region's start event
            prefetch(0)
        if i + 1 < args.steps:
            prefetch(i + 1)
        b = i % 2
        torch.cuda.current_stream(dev).wait_event(loaded[b])
        v = step_fn(i, bufs[b][0], bufs[b][1])
        consumed[b].record(torch.cuda.current_stream(dev))
        out_host[i % n_batches].copy_(v, non_blocking=True)
    ms_e2e = max_over_ranks(timed_loop(e2e_step, args.steps, world)[0], world)
    e2e_tok_s = N * world / (ms_e2e / args.steps / 1e3)

    # roofline of the dominant kernel: lazy Adam over the U touched rows of a (rows, 384) fp32 table
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    hbm = peaks.get("hbm_gbs")
    peak_src = "measured" if hbm else "fallback"
    hbm = hbm or 6650.0
    adam_ms = statistics.mean(per_kernel["lazy_adam_step"])
    M = N * HEADS * KNN
    # one backward per step: the row sums go straight into the step (one GPU, or shards behind the peer exchange)
    fused = mem.shard is None or mem.shard_exchange == "p2p"
    if fused:
        # the fused step: read p / m / v and write them back for every touched row, clear its mark, read the
        # sorted (row, position) pairs and weights and the output gradient rows (the accumulator is never used)
        adam_bytes = U * D_MODEL * 4 * 6 + U + M * 12 + N * D_MODEL * 4
    else:
        # mask scan, row list, read p / m / v / acc, write p / m / v (the clean RowStore keeps consumed acc rows)
        adam_bytes = rows * 1 + U * (4 + 4 + 1) + U * D_MODEL * 4 * 7
    roof = {"kernel": "lazy_adam_step (fused with the deferred row sums)" if fused else "lazy_adam_step",
            "bound": "hbm", "achieved": adam_bytes / (adam_ms / 1e3) / 1e9,
            "peak": hbm, "peak_source": peak_src, "unit": "GB/s",
            "traffic": round((ADAM_TRAFFIC_PER_ROW if fused else ADAM_UNFUSED_TRAFFIC_PER_ROW) * U),
            "traffic_source": "ncu dram bytes per touched row on a 1M-row capture, scaled by the measured rows",
            "algorithmic_bytes": adam_bytes, "unique_rows": U}
    roof["frac"] = roof["achieved"] / roof["peak"]
    kernel_bytes = {
        "bag_forward": M * (D_MODEL * 4 + 12) + N * D_MODEL * 4,
        # the weight gradient alone: every lookup's table row, its index and weight, grad_out, gw written
        "bag_weight_grad": M * (D_MODEL * 4 + 8 + 4 + 4) + N * D_MODEL * 4,
        # the rest of the backward: key build and sort (2 passes of keys and positions), then the norm pass
        # (sorted pairs, weights, grad_out, row norms and marks); without the fused step also the rows written
        "bag_backward_rows": M * (8 * 4 + 4) + N * D_MODEL * 4 + U * 5 + (0 if fused else U * D_MODEL * 4),
        "lazy_adam_step": adam_bytes,
        # row-sharded owner side: every rank's lookups scanned (8 B), this shard's ~M rows gathered, partials out
        "shard_bag_forward": world * M * 8 + M * D_MODEL * 4 + world * N * D_MODEL * 4,
        "shard_bag_backward_rows": (U * D_MODEL * 4 * (0 if fused else 1) + world * M * (8 * 4 + 8)
                                    + world * N * D_MODEL * 4 + U * 5),
    }
    # the fused scoring + selection: its sub-key contraction on the tensor cores (algorithmic FLOPs) against the
    # measured bf16 GEMM burst peak; the selection in its epilogue and the pair kernel share the same time
    kernel_flops = {"score_select": 2 * N * HEADS * 2 * n_keys * (K_DIM // 2)}
    tc_peak = peaks.get("bf16_tflops") or 1590.0
    breakdown = {}
    for name, t in sorted(per_kernel.items()):
        entry = {"ms": round(statistics.mean(t), 4), "calls_per_step": len(t) / args.steps}
        if name in kernel_bytes:
            gbs = kernel_bytes[name] / (statistics.mean(t) / 1e3) / 1e9
            entry.update({"GB/s": round(gbs, 1), "frac": round(gbs / hbm, 3)})
        if name in kernel_flops:
            tfs = kernel_flops[name] / (statistics.mean(t) / 1e3) / 1e12
            entry.update({"TFLOP/s": round(tfs, 1), "tensor_frac": round(tfs / tc_peak, 3)})
        breakdown[name] = entry

    line = {"metric": METRIC, "value": round(tokens_per_s, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "pkm-layer-b16m" if n_keys == 4096 else f"pkm-layer-{n_keys ** 2}rows",
                       "rows": n_keys ** 2, "rows_per_gpu": rows, "rows_per_half": n_keys, "v_dim": D_MODEL, "heads": HEADS, "knn": KNN,
                       "k_dim": K_DIM, "tokens_per_gpu": N, "global_tokens": N * world,
                       "scoring": "bf16 autocast (bf16 operands, fp32 accumulate)", "values": "fp32 table",
                       "optimizer": "LazyRowAdam fp32 moments + fused AdamW (dense)",
                       "parallelism": f"dp{world} tokens + {world}-way row-sharded table" if world > 1 else "single",
                       "l2": "working set > L2: each step gathers ~6.4 GB of table rows and updates ~U rows of "
                             "table + moments (77 GB resident), inputs cycle over 4 batches",
                       "unique_rows_per_step_per_gpu": round(U)},
            "e2e": {"value": round(e2e_tok_s, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 2 * N * D_MODEL * 4, "d2h_bytes_per_step": 4,
                    "note": "a training step: the inputs (activations and upstream gradient) go in every step; "
                            "only the step's scalar (the value clip norm) comes back, the layer output and the "
                            "updated rows stay on the device"},
            "gpu_launches": launches, "host_ms_per_step": round(host_ms / args.steps, 4),
            "step_mode": ("one CUDA graph per step (smlm_b200.graph_step.GraphedStep; inputs copied into its static "
                          "buffers every step)" if graphed else "eager calls"),
            "eager": {"ms_per_step": round(eager_ms / args.steps, 4),
                      "host_ms_per_step": round(eager_host_ms / args.steps, 4),
                      "tokens_per_s": round(N * world / (eager_ms / args.steps / 1e3), 1)},
            "kernel_timing": "per-call CUDA events on the launching stream over K further identical eager steps",
            "roofline": roof, "kernels": breakdown, "clocks": clocks.summary()}
    if world > 1:
        try:
            xr = exchange_rooflines({name: statistics.mean(t) for name, t in per_kernel.items()}, world, N,
                                    HEADS * KNN, D_MODEL, hbm)
            line["exchange"] = {"peak_nvlink_gbs": NVLINK_PEER_GBS,
                                "peak_source": "measured peer copy per direction per GPU on this pool (nominal 900)",
                                "calls": xr,
                                "nccl_allgather_bytes_in_per_step": (world - 1) * N * D_MODEL * 4}
        except (KeyError, TypeError, ValueError, ZeroDivisionError) as exc:
            # a report of the measured calls: its failure is shown in the line, the measurement stands
            line["exchange"] = {"error": repr(exc)}
    if graphed:
        del gstep, step_fn                  # a graph holding NCCL calls is released before the process group
    if world > 1:
        torch.cuda.synchronize(dev)
        x = getattr(mem.values.weight, "peer_exchange", None)
        if x is not None:
            x.close()
    return line


# -------------------------------------------------------------------------------------- configs 1 - 4
# name, sub-keys per half, tokens per step, bf16 autocast, BatchNorm query + swilu, table optimizer, layer input
# ("gauss": x ~ N(0, 1); "zipf": x = a random N(0, 1) embedding of token ids drawn half uniform, half Zipf(1.1)
# over a 50,304-id vocabulary, so that frequent tokens make hot rows), bf16 value copy read by the forward
LAYER_CONFIGS = [
    ("config1-layer-65k-fp32", 256, 2048, False, False, "adam", "gauss", False),
    ("config2-b1m-layer", 1024, 32768, True, True, "adam", "gauss", False),
    ("config2-b1m-layer-bf16-values", 1024, 32768, True, True, "adam", "gauss", True),
    ("config2-b1m-layer-bf16-moments", 1024, 32768, True, True, "adam-bf16", "gauss", False),
    ("config3-b4m-layer-rowrms", 2048, 65536, True, True, "rowrms", "gauss", False),
    ("config4-b16m-layer-zipf", 4096, 32768, True, False, "adam", "zipf", False),
    ("config4-b16m-layer-zipf-bf16-values", 4096, 32768, True, False, "adam", "zipf", True),
]
ZIPF_VOCAB, ZIPF_S = 50304, 1.1


def zipf_mix_tokens(n, gen, device):
    """n token ids: half uniform over ZIPF_VOCAB, half Zipf(ZIPF_S) over the ranks (id = rank - 1), shuffled."""
    rank = torch.arange(1, ZIPF_VOCAB + 1, dtype=torch.float64, device=device)
    p = rank ** -ZIPF_S
    zipf = torch.multinomial((p / p.sum()).float(), n - n // 2, replacement=True, generator=gen)
    uni = torch.randint(0, ZIPF_VOCAB, (n // 2,), device=device, generator=gen)
    mix = torch.cat([uni, zipf])
    return mix[torch.randperm(n, device=device, generator=gen)]


def layer_inputs(kind, N, gen, device):
    if kind == "gauss":
        return torch.randn(N, D_MODEL, device=device, generator=gen)
    emb = getattr(layer_inputs, "emb", None)
    if emb is None or emb.device != device:
        emb = layer_inputs.emb = torch.randn(ZIPF_VOCAB, D_MODEL, device=device, generator=gen)
    return emb[zipf_mix_tokens(N, gen, device)]


def run_configs(args):
    """BASELINE configs 1-4 as single PKM layers on one GPU, each phase device-timed: config 1 (65,536 rows,
    2,048 tokens, fp32 without autocast, no BatchNorm / swilu, LazyRowAdam), config 2 (the B-1M model's layer:
    1,048,576 rows, 32 x 1024 tokens, bf16 autocast, BatchNorm query and swilu, LazyRowAdam with fp32 moments, with
    the forward reading a bf16 copy of the fp32 master (the config's "values bf16 with fp32 master"), and with bf16
    moments), config 3 (the B-4M layer: 4,194,304 rows, 64 x 1024 tokens, the row-wise rowrms optimizer), config 4
    (the B-16M layer, 32 x 1024 tokens per GPU, its inputs embeddings of a uniform + Zipf(1.1) token mix: hot
    rows). Seeded synthetic inputs, upstream gradient ~ N(0, 1). fwd = the layer's forward; bwd = backward +
    value / dense clipping; opt = the table optimizer + fused AdamW on the dense parameters (with deferred row sums
    the table's row sums run in opt, not in bwd). The fp32 lazy-Adam configurations are also timed as one CUDA
    graph per step (GraphedStep, captured first; `graphed_step_ms`), which removes the host's launch time that
    bounds the small configurations' eager steps."""
    from smlm_b200.pkm import ProductKeyMemory
    from smlm_b200.row_optim import RowWiseOptimizer
    from smlm_b200.sparse_values import LazyRowAdam, OptimizerSet, clip_row_sparse, row_store
    dev = torch.device("cuda", 0)
    out = []
    for name, n_keys, N, autocast, bn, kind, inputs, copy in LAYER_CONFIGS:
        torch.manual_seed(0)
        with torch.device(dev):
            mem = ProductKeyMemory(D_MODEL, D_MODEL, n_keys=n_keys, heads=HEADS, knn=KNN, k_dim=K_DIM,
                                   query_norm="batchnorm" if bn else "none", swilu=bn, value_grad="row_sparse")
            if not bn:   # config-1 initialisation
                with torch.no_grad():
                    mem.query_proj.weight.normal_(0, 0.02)
                    mem.keys.normal_(0, (K_DIM // 2) ** -0.5)
        table = mem.values.weight
        dense = [p for p in mem.parameters() if p is not table]
        graphed = kind == "adam"            # fp32 lazy Adam: the whole step also as one CUDA graph
        if kind == "rowrms":
            topt = RowWiseOptimizer([table], lr=1e-3, kind="rowrms", beta2=0.98)
        else:
            topt = LazyRowAdam([table], lr=1e-3, betas=(0.9, 0.98), eps=1e-8,
                               state_dtype="bf16" if kind == "adam-bf16" else "fp32",
                               value_copy_dtype=torch.bfloat16 if copy else None, capturable=graphed)
        opt = OptimizerSet(torch.optim.AdamW(dense, lr=1e-3, betas=(0.9, 0.98), weight_decay=0.0, fused=True,
                                             capturable=graphed), topt)
        gen = torch.Generator(device=dev).manual_seed(1)
        xs = [layer_inputs(inputs, N, gen, dev) for _ in range(2)]
        gs = [torch.randn(N, D_MODEL, device=dev, generator=gen) for _ in range(2)]
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
        uniq = []
        graph_ms = None
        if graphed:
            # captured before any eager step (autograd's gradient streams), then replayed on alternating inputs
            from smlm_b200.graph_step import GraphedStep

            def whole(x, g):
                with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
                    o = mem(x)
                o.backward(g)
                vnorm = clip_row_sparse([table], 1.0)
                torch.nn.utils.clip_grad_norm_([p for p in dense if p.grad is not None], 1.0, foreach=True)
                opt.step()
                opt.zero_grad(set_to_none=True)
                return vnorm
            gstep = GraphedStep(whole, [xs[0], gs[0]], opt.opts, warmup=max(3, args.warmup))
            for i in range(args.warmup):
                gstep(xs[i % 2], gs[i % 2])
            torch.cuda.synchronize()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record()
            for i in range(args.steps):
                gstep(xs[i % 2], gs[i % 2])
            g1.record()
            torch.cuda.synchronize()
            graph_ms = g0.elapsed_time(g1) / args.steps
            del gstep

        def step(i, e=None):
            if e:
                e[0].record()
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
                o = mem(xs[i % 2])
            if e:
                e[1].record()
            o.backward(gs[i % 2])
            clip_row_sparse([table], 1.0)
            torch.nn.utils.clip_grad_norm_([p for p in dense if p.grad is not None], 1.0, foreach=True)
            if e:
                e[2].record()
            else:
                uniq.append(row_store(table).touched_rows())
            opt.step()
            opt.zero_grad(set_to_none=True)
            if e:
                e[3].record()
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        for i in range(args.steps):
            step(i, ev[i])
        torch.cuda.synchronize()
        ph = [sum(e[j].elapsed_time(e[j + 1]) for e in ev) / args.steps for j in range(3)]
        entry = {"config": name, "rows": n_keys ** 2, "tokens": N, "autocast_bf16": autocast,
                 "query_norm_swilu": bn, "optimizer": kind, "inputs": inputs,
                 "values_read": "bf16 copy of the fp32 master" if copy else "fp32 table",
                 "fwd_ms": round(ph[0], 4), "bwd_ms": round(ph[1], 4), "opt_ms": round(ph[2], 4),
                 "tokens_per_s": round(N / (sum(ph) / 1e3), 1),
                 "graphed_step_ms": round(graph_ms, 4) if graph_ms is not None else None,
                 "graphed_tokens_per_s": round(N / (graph_ms / 1e3), 1) if graph_ms is not None else None,
                 "unique_rows_per_step": round(sum(uniq[1:]) / max(1, len(uniq) - 1))}
        if inputs == "zipf":
            with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
                mem.record = True
                mem(xs[0])
                mem.record = False
            _, counts = torch.unique(mem.last_indices, return_counts=True)
            entry["max_lookups_per_row"] = int(counts.max())
            entry["lookups_on_rows_read_over_64_times"] = round(float(counts[counts > 64].sum() / counts.sum()), 4)
        out.append(entry)
        del mem, opt, topt, xs, gs
        import gc
        gc.collect()
        torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------------------- config 2 model
def run_model_case(args):
    """BASELINE configs[1], the B-1M training step on one GPU: a 6-layer model (d_model 384, 6 attention heads,
    SwiGLU 1024, vocab 32,768 with the embedding tied to the LM head, RMSNorm, RoPE), the product-key memory in
    place of the feed-forward of layer 3 (0-based: the fourth block; 1024 sub-keys per half, 1,048,576 rows x 384,
    BatchNorm query and swilu), values bf16 with an fp32 master (the forward reads the bf16 copy), 32 x 1024 tokens
    uniform over the vocabulary per step, next-token cross entropy, bf16 autocast, clipping as the reference's
    training loop does (values and the rest separately to 1.0), LazyRowAdam on the table and fused AdamW (weight
    decay 0.1) on the rest. Random-init weights, seeded synthetic tokens. Timed as the whole step replayed as one
    CUDA graph and as eager calls with fwd / bwd / opt separated (CUDA events)."""
    from smlm_b200.graph_step import GraphedStep
    from smlm_b200.model import ModelConfig, Transformer
    from smlm_b200.optim import build_optimizer, clip_grads
    from smlm_b200.sparse_values import row_sparse_tables, row_store
    dev = torch.device("cuda", 0)
    B, T, vocab = 32, 1024, 32768
    cfg = ModelConfig(vocab_size=vocab, d_model=D_MODEL, n_layers=6, n_heads=6, ffn_hidden=1024, max_seq_len=T,
                      mem_layers=[3], mem_n_keys=1024, mem_value_grad="row_sparse")
    torch.manual_seed(0)
    with torch.device(dev):
        model = Transformer(cfg)
    opt = build_optimizer(model, lr=1e-3, value_lr=1e-3, weight_decay=0.1, betas=(0.9, 0.95),
                          value_copy_dtype=torch.bfloat16, capturable=True)
    gen = torch.Generator(device=dev).manual_seed(2)
    seqs = [torch.randint(0, vocab, (B, T + 1), device=dev, generator=gen) for _ in range(4)]
    batches = [(s[:, :-1].contiguous(), s[:, 1:].contiguous()) for s in seqs]

    def forward(ids, tgt):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            _, loss = model(ids, targets=tgt)
        return loss

    def finish(loss):
        loss.backward()
        clip_grads(model, 1.0)

    def step(ids, tgt):
        loss = forward(ids, tgt)
        finish(loss)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss.detach()

    # captured first (autograd binds each parameter's gradient accumulation to the stream of its first backward)
    gstep = GraphedStep(step, list(batches[0]), opt.opts, warmup=max(3, args.warmup))
    for i in range(args.warmup):
        gstep(*batches[i % 4])
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clocks:
        s.record()
        for i in range(args.steps):
            gstep(*batches[i % 4])
        e.record()
        torch.cuda.synchronize()
    graph_ms = s.elapsed_time(e) / args.steps
    loss_now = float(gstep.outputs)
    # eager phases (the optimizers keep stepping: same work per step); LazyRowAdam(capturable=True) runs its
    # eager steps through the same fused kernel
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    table = row_sparse_tables(model)[0]
    uniq = []
    for i in range(args.steps + 1):
        e4 = ev[i - 1] if i else None
        ids, tgt = batches[i % 4]
        if e4:
            e4[0].record()
        loss = forward(ids, tgt)
        if e4:
            e4[1].record()
        finish(loss)
        if e4:
            e4[2].record()
        else:
            uniq.append(row_store(table).touched_rows())
        opt.step()
        opt.zero_grad(set_to_none=True)
        if e4:
            e4[3].record()
    torch.cuda.synchronize()
    ph = [sum(x[j].elapsed_time(x[j + 1]) for x in ev) / args.steps for j in range(3)]
    return {"case": "model", "config": "config2-b1m-model",
            "model": "6 layers, d_model 384, 6 heads, SwiGLU 1024, vocab 32768 tied, PKM (1024^2 rows x 384, "
                     "BatchNorm query, swilu) in place of the FFN of layer 3 (0-based)",
            "values": "bf16 copy read by the forward, fp32 master and fp32 Adam moments (LazyRowAdam)",
            "tokens_per_step": B * T, "steps": args.steps, "warmup": args.warmup,
            "graph_ms_per_step": round(graph_ms, 4), "tokens_per_s": round(B * T / (graph_ms / 1e3), 1),
            "eager": {"fwd_ms": round(ph[0], 4), "bwd_ms": round(ph[1], 4), "opt_ms": round(ph[2], 4),
                      "tokens_per_s": round(B * T / (sum(ph) / 1e3), 1)},
            "loss_after_warmup_and_timed_steps": round(loss_now, 4),
            "unique_rows_per_step": uniq[0] if uniq else None, "clocks": clocks.summary()}


# ------------------------------------------------------------------------------------------- B-16M model step
def run_model_b16m(args):
    """The reference's B-16M-sparse training step on one GPU (its `smlm/train.py` preset and its own long run's
    settings: 12 layers, d_model 384, 6 heads, SwiGLU 1024, vocab 50,304 tied, memory layers 2 / 6 / 10 sharing one
    4096^2 = 16,777,216 x 384 fp32 table with BatchNorm queries and swilu, row-sparse gradients, LazyRowAdam with
    fp32 moments at value lr 2.4e-3 and fused AdamW (lr 6e-4, betas 0.9 / 0.95, weight decay 0.1) on the rest,
    values and the rest clipped separately to 1.0, bf16 autocast, 32 sequences x 1024 tokens per step uniform over
    the vocabulary, next-token cross entropy; random-init weights, seeded synthetic tokens). --impl cuda runs this
    build's modules, --impl reference the reference's own `smlm` package (vendored unmodified in baseline/_ref)
    with its Triton memory kernels, on the same GPU. --micro-batch sets the sequences per forward (the gradients of
    the step's micro-batches accumulate, loss / accum each, as the reference's loop does; its long run used 4).
    This build's step is captured as one CUDA graph (GraphedStep; its eager time beside it), the reference's runs
    eagerly: CUDA events around --steps consecutive steps after --warmup."""
    dev = torch.device("cuda", 0)
    B, T, vocab = 32, 1024, 50304
    mb = args.micro_batch or B
    if B % mb:
        raise ValueError("--micro-batch must divide 32")
    accum = B // mb
    if args.impl == "reference":
        if not os.path.isfile(os.path.join(REF_PKG, "smlm", "model.py")):
            return {"case": "model", "impl": "reference", "unavailable": "the reference package is not in "
                    "baseline/_ref (build it with __graft_entry__.build())"}
        if REF_PKG not in sys.path:
            sys.path.insert(0, REF_PKG)
        from smlm.model import ModelConfig, Transformer
        from smlm.optim import build_optimizer, clip_grads
        extra = dict(mem_impl="triton")
        what = "the reference's smlm package (baseline/_ref, unmodified), mem_impl=triton"
    else:
        from smlm_b200.model import ModelConfig, Transformer
        from smlm_b200.optim import build_optimizer, clip_grads
        extra = {}
        what = "this build (smlm_b200)"
    cfg = ModelConfig(vocab_size=vocab, d_model=D_MODEL, n_layers=12, n_heads=6, ffn_hidden=1024, max_seq_len=T,
                      mem_layers=[2, 6, 10], mem_n_keys=4096, mem_share_values=True, mem_value_grad="row_sparse",
                      **extra)
    torch.manual_seed(0)
    with torch.device(dev):
        model = Transformer(cfg)
    model.train()
    graphed = args.impl == "cuda"       # this build captures the whole step (LazyRowAdam(capturable=True))
    opt = build_optimizer(model, lr=6e-4, value_lr=2.4e-3, weight_decay=0.1, betas=(0.9, 0.95),
                          **({"capturable": True} if graphed else {}))
    gen = torch.Generator(device=dev).manual_seed(2)
    seqs = [torch.randint(0, vocab, (B, T + 1), device=dev, generator=gen) for _ in range(2)]

    def train(s_):
        loss_sum = torch.zeros((), device=dev)
        for a in range(accum):
            x = s_[a * mb:(a + 1) * mb]
            with torch.autocast("cuda", dtype=torch.bfloat16):
                _, loss = model(x[:, :-1], x[:, 1:])
            (loss / accum).backward()
            loss_sum += loss.detach() / accum
        clip_grads(model, 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss_sum

    def timed(step):
        for i in range(args.warmup):
            step(seqs[i % 2])
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(0) as clocks:
            s.record()
            for i in range(args.warmup, args.warmup + args.steps):
                loss = step(seqs[i % 2])
            e.record()
            torch.cuda.synchronize()
        return s.elapsed_time(e) / args.steps, float(loss), clocks.summary()

    eager_ms = None
    if graphed:
        # captured first (autograd binds each parameter's gradient accumulation to the stream of its first backward)
        from smlm_b200.graph_step import GraphedStep
        gstep = GraphedStep(train, [seqs[0]], opt.opts, warmup=max(3, args.warmup))
        ms, loss, clocks = timed(gstep)
        del gstep
        eager_ms, _, _ = timed(train)
    else:
        ms, loss, clocks = timed(train)
    return {"case": "model", "config": "b16m-model-train", "impl": args.impl, "what": what,
            "step_mode": "one CUDA graph per step (GraphedStep)" if graphed else "eager",
            "eager_ms_per_step": round(eager_ms, 3) if eager_ms is not None else None,
            "model": "B-16M-sparse: 12 layers, d_model 384, 6 heads, SwiGLU 1024, vocab 50304 tied, PKM in layers "
                     "2/6/10 sharing one 4096^2 x 384 fp32 table (BatchNorm query, swilu), LazyRowAdam fp32",
            "tokens_per_step": B * T, "micro_batch": mb, "grad_accum": accum, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "tokens_per_s": round(B * T / (ms / 1e3), 1),
            "loss": round(loss, 4), "peak_gib": round(torch.cuda.max_memory_allocated(dev) / 2**30, 1),
            "clocks": clocks,
            "reference_published": "138.0k tok/s on an H200 NVL (its long B-16M run, micro-batch 4, Triton kernels)"}


# ------------------------------------------------------------------------------------------------ engram
def run_engram(args):
    """The reference's default Engram n-gram memory module on one GPU (orders 2 and 3, 8 hash heads each, rows of
    24 values, 524,287 rows per head: a 8,388,592 x 24 fp32 table), d_model 384, 32 x 1024 seeded uniform token
    ids per step (used as compressed ids: the GPT-2 token compression needs tiktoken's vocabulary, not available
    offline), hidden states and upstream gradient ~ N(0, 1). One step = the hash of every position (ngram_rows),
    the module's forward (16 one-lookup value bags, gating, RMSNorms, depthwise convolution), backward into the
    row store, value clipping, LazyRowAdam on the table and fused AdamW on the dense parts. Device-timed with CUDA
    events (whole step, and per library call over as many further steps)."""
    from smlm_b200 import _lib as L
    from smlm_b200.engram import EngramMemory, NgramHash
    from smlm_b200.sparse_values import LazyRowAdam, OptimizerSet, clip_row_sparse
    dev = torch.device("cuda", 0)
    B, T, vocab = 32, 1024, 32768
    orders, heads, hd, rows = (2, 3), 8, 24, 524287
    torch.manual_seed(0)
    ng = NgramHash(vocab, orders, heads, rows, seed=0, canon=(torch.arange(vocab), vocab)).to(dev)
    with torch.device(dev):
        mod = EngramMemory(D_MODEL, ng.n_lookups, hd, rows, conv_kernel=4, dilation=max(orders))
    table = mod.values.weight
    dense = [p for p in mod.parameters() if p is not table]
    opt = OptimizerSet(torch.optim.AdamW(dense, lr=1e-3, betas=(0.9, 0.98), weight_decay=0.0, fused=True),
                       LazyRowAdam([table], lr=1e-3, betas=(0.9, 0.98), eps=1e-8))
    gen = torch.Generator(device=dev).manual_seed(3)
    ids = [torch.randint(0, vocab, (B, ng.history + T), device=dev, generator=gen) for _ in range(2)]
    hs = [torch.randn(B, T, D_MODEL, device=dev, generator=gen) for _ in range(2)]
    gs = [torch.randn(B, T, D_MODEL, device=dev, generator=gen) for _ in range(2)]

    def step(i):
        r = ng(ids[i % 2])
        y = mod(hs[i % 2], r)
        y.backward(gs[i % 2])
        clip_row_sparse([table], 1.0)
        torch.nn.utils.clip_grad_norm_([p for p in dense if p.grad is not None], 1.0, foreach=True)
        opt.step()
        opt.zero_grad(set_to_none=True)

    for i in range(args.warmup):
        step(i)
    uniq = int(torch.unique(ng(ids[0])).numel())                    # distinct rows one step reads
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        step(i)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    L.PROFILE = []
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    prof, L.PROFILE = L.PROFILE, None
    per = {}
    for name, a, b, _ in prof:
        per.setdefault(name, []).append(a.elapsed_time(b))
    lookups = B * T * ng.n_lookups
    return {"case": "engram", "module": "EngramMemory(d_model 384, orders 2/3 x 8 heads, 24-value rows, "
                                       "524,287 rows per head)", "table_rows": table.shape[0], "tokens": B * T,
            "lookups_per_step": lookups, "unique_rows_per_step": uniq, "steps": args.steps,
            "ms_per_step": round(ms, 4), "tokens_per_s": round(B * T / (ms / 1e3), 1),
            "kernels": {k: {"ms": round(statistics.mean(v), 4), "calls_per_step": len(v) / args.steps}
                        for k, v in sorted(per.items())}}


# ------------------------------------------------------------------------------------------- host-RAM tables
# (name, table optimizer, GACC, HOT fraction): the reference's host-table configurations (its step-21 benchmark)
HOST_CONFIGS = (("adam", "adam", False, 0.0), ("rowrms", "rowrms", False, 0.0), ("rowrms+gacc", "rowrms", True, 0.0),
                ("rowrms+hot5%+gacc", "rowrms", True, 0.05))


def _mem_available():
    try:
        return [int(ln.split()[1]) * 1024 for ln in open("/proc/meminfo") if ln.startswith("MemAvailable")][0]
    except (OSError, IndexError):
        return 0


def _host_link_gbs(dev, nbytes=1 << 30):
    """Pinned host <-> device copy bandwidth (GB/s) of this box, each direction: the denominators of the host path."""
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = {}
    for name, fn in (("h2d", lambda: d.copy_(h, non_blocking=True)), ("d2h", lambda: h.copy_(d, non_blocking=True))):
        fn()
        out[name] = round(3 * nbytes / 1e9 / (_event_ms(fn, 3) / 1e3), 1)
    return out


def _host_layer(PKM, n_keys, table):
    """The B-16M layer (config-1 layer: no BatchNorm / swilu) built on the meta device, its dense parameters then
    materialised on the CPU with the config-1 initialisation (seed 0) and its value table set to `table` (a host
    tensor shared by every configuration, so the 25.8 GB table is filled once)."""
    from torch import nn
    with torch.device("meta"):
        mem = PKM(d_in=D_MODEL, d_out=D_MODEL, n_keys=n_keys, heads=HEADS, knn=KNN, k_dim=K_DIM,
                  query_norm="none", swilu=False, value_grad="row_sparse")
    mem.values.weight = nn.Parameter(table)
    for mod in mem.modules():
        for name, p in list(mod._parameters.items()):
            if p is not None and p.is_meta:
                mod._parameters[name] = nn.Parameter(torch.empty(p.shape, dtype=p.dtype), p.requires_grad)
        for name, b in list(mod._buffers.items()):
            if b is not None and b.is_meta:
                mod._buffers[name] = torch.zeros(b.shape, dtype=b.dtype)
    torch.manual_seed(0)
    with torch.no_grad():
        mem.query_proj.weight.normal_(0, 0.02)
        mem.query_proj.bias.zero_()
        mem.keys.normal_(0, (K_DIM // 2) ** -0.5)
    return mem


def _host_arm(ours):
    """The host-table modules of one arm: this build's smlm_b200, or the reference's own smlm package as vendored,
    unmodified, into baseline/_ref (None when it is absent)."""
    if ours:
        from smlm_b200 import host_optim, host_values, pkm, row_optim, sparse_values
        return dict(PKM=pkm.ProductKeyMemory, hv=host_values, Adam=host_optim.HostLazyRowAdam,
                    Row=row_optim.RowWiseOptimizer, clip=sparse_values.clip_row_sparse,
                    row_store=sparse_values.row_store)
    if not os.path.isfile(os.path.join(REF_PKG, "smlm", "host_values.py")):
        return None
    if REF_PKG not in sys.path:
        sys.path.insert(0, REF_PKG)
    from smlm import host_optim, host_values, pkm, row_optim, sparse_values
    return dict(PKM=lambda **kw: pkm.ProductKeyMemory(impl="torch", **kw), hv=host_values,
                Adam=host_optim.HostLazyRowAdam, Row=row_optim.RowWiseOptimizer, clip=sparse_values.clip_row_sparse,
                row_store=sparse_values.row_store)


def _host_config(arm, ours, config, table, n_keys, xs, gs, reads, capacity, dev, steps, warmup):
    """One configuration of one arm: the layer step (bf16 autocast forward, backward, value clipping, the table
    optimizer, fused AdamW on the dense parameters) with the table in host RAM; wall time per step with the device
    synchronised on both sides of `steps` consecutive steps after `warmup`, then one more step with the staging
    phases timed (host_timings)."""
    name, optim, gacc, hot = config
    mem = _host_layer(arm["PKM"], n_keys, table)
    arm["hv"].enable_host_values(mem)
    mem.to(dev)
    weight = mem.values.weight
    if hot:
        arm["hv"].enable_hot_rows(mem, reads, hot, dev)
    if gacc:
        # this build's step accumulator writes the updated rows back while the next step runs (overlap)
        arm["hv"].enable_step_rows(mem, capacity, dev, **({"overlap": True} if ours else {}))
    dense = [p for p in mem.parameters() if p is not weight]
    adamw = torch.optim.AdamW(dense, lr=1e-3, betas=(0.9, 0.98), weight_decay=0.0, fused=True)
    topt = (arm["Adam"]([weight], lr=1e-3, betas=(0.9, 0.98), eps=1e-8) if optim == "adam"
            else arm["Row"]([weight], lr=2.4e-3, kind="rowrms"))

    def step(i):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = mem(xs[i % 2])
        out.backward(gs[i % 2])
        arm["clip"]([weight], 1.0)
        torch.nn.utils.clip_grad_norm_([p for p in dense if p.grad is not None], 1.0, foreach=True)
        adamw.step()
        topt.step()
        adamw.zero_grad(set_to_none=True)
        topt.zero_grad(set_to_none=True)

    # the steps alternate the two input batches throughout (warm-up, timed, profiled), so every timed step reads
    # the rows of the other batch after its predecessor, as in training on fresh data
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(warmup, warmup + steps):
        step(i)
    torch.cuda.synchronize()                       # every stream: the last write-back is inside the time
    dt = (time.perf_counter() - t0) / steps
    arm["hv"].host_timings(mem, reset=True)
    mem.values.profile = True
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    step(warmup + steps)
    torch.cuda.synchronize()
    profiled = time.perf_counter() - t0
    phases = arm["hv"].host_timings(mem, reset=True)
    mem.values.profile = False
    res = {"ms_per_step": round(dt * 1e3, 1), "tokens_per_s": round(xs[0].shape[0] / dt, 1),
           "profiled_step_ms": round(profiled * 1e3, 1),
           "phases_ms": {k: round(v * 1e3, 1) for k, v in phases.items()}}
    if gacc:
        res["gacc_peak_rows"] = int(mem.values.step_rows.peak)
        res["gacc_spilled_steps"] = int(mem.values.step_rows.spilled_steps)
    # drop everything this configuration allocated on the host before the next one (the shared table stays)
    st = getattr(weight, "row_store", None)
    if ours:
        state = topt.state.get(weight, {})
        arm["hv"].release(*[v for v in state.values() if torch.is_tensor(v)],
                          getattr(st, "_acc", None), getattr(st, "touched", None))
    del mem, adamw, topt, weight, st, step
    import gc
    gc.collect()
    torch.cuda.empty_cache()
    return res


def run_host(args):
    """BASELINE config 4's layer (--rows-per-half 4096: 16,777,216 x 384 fp32 table; 32,768 tokens per step, the
    bench's default workload) with the value table in host RAM, one GPU: the reference's host-table configurations (Adam, rowrms,
    rowrms + GACC, rowrms + HOT 5% + GACC) through this build's smlm_b200.host_values and, on the same box and
    inputs, through the reference's own smlm.host_values (its C row loops on the host cores, stock PyTorch on the
    GPU). HOT ranks rows by the read counts of the timed inputs (the best case, as the reference's own benchmark
    of it). A configuration whose host RAM would not fit (with 16 GB to spare) is skipped.

    `host_link` is this build's roofline: the table rows that must cross the host link per step, in each direction,
    as multiples of the distinct rows U (Adam: in = gather + the update's p, m, v, accumulator = 5, out = the add's
    accumulator rows (a step's first add writes them without reading) + p, m, v = 4, the clip norm from the rows'
    squared norms that the add kept on the GPU; rowrms: 3 in, 2 out, its row state on the GPU; GACC: in = the rows the previous step
    did not read (the others come from the device cache), out = the updated rows; HOT rows never cross), over the
    measured pinned copy bandwidths: serial_ms one direction after the other, duplex_ms both at once (this build's
    GACC step overlaps its write-back with the next step); frac = serial_ms / the measured step (above 1 only
    through overlap)."""
    from smlm_b200.pkm import ProductKeyMemory as OurPKM
    dev = torch.device("cuda", 0)
    n_keys, N = args.rows_per_half, args.tokens
    rows = n_keys ** 2
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    table = torch.empty(rows, D_MODEL, dtype=torch.float32)
    gen = torch.Generator(device=dev).manual_seed(11)
    chunk = 1 << 20
    for a in range(0, rows, chunk):                     # N(0, 384^-0.5), generated on the GPU in 1M-row chunks
        table[a:a + chunk].copy_(torch.randn(min(chunk, rows - a), D_MODEL, device=dev, generator=gen)
                                 * D_MODEL ** -0.5)
    xs = [torch.randn(N, D_MODEL, device=dev, generator=gen) for _ in range(2)]
    gs = [torch.randn(N, D_MODEL, device=dev, generator=gen) for _ in range(2)]
    # read counts and distinct rows per step of the timed inputs, from the layer's own selection
    # (the query projection and the selection of the same layer: same seed, so the rows the timed steps' first
    # forwards read)
    probe = _host_layer(OurPKM, n_keys, torch.empty(1, D_MODEL))
    probe.query_proj.to(dev)
    keys = probe.keys.detach().to(dev)
    reads = torch.zeros(rows, dtype=torch.int64, device=dev)
    distinct, read_sets = [], []
    from smlm_b200 import kernels as K
    with torch.no_grad():
        for x in xs:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                q = probe.query_proj.to(dev)(x).view(N, HEADS, K_DIM)
            _, idx, _ = K.score_select(q.bfloat16(), keys.bfloat16(), KNN)
            reads += torch.bincount(idx.reshape(-1), minlength=rows)
            distinct.append(int(torch.unique(idx).numel()))
            read_set = torch.zeros(rows, dtype=torch.bool, device=dev)
            read_set[idx.reshape(-1)] = True
            read_sets.append(read_set)
    del probe, keys
    capacity = int(max(distinct) * 1.05)
    hot_rows = int(round(0.05 * rows))
    hot_share = float(reads.sort(descending=True).values[:hot_rows].sum() / reads.sum())
    is_hot = torch.zeros(rows, dtype=torch.bool, device=dev)
    is_hot[torch.argsort(reads, descending=True, stable=True)[:hot_rows]] = True
    # (rows in host RAM one step reads, of which the previous step read too): the timed steps alternate the inputs
    both = read_sets[0] & read_sets[1]
    plain_cold = (distinct[0], int(both.sum()))
    hot_cold = (int((read_sets[0] & ~is_hot).sum()), int((both & ~is_hot).sum()))
    del read_sets, both, is_hot
    reads = reads.cpu()
    link = _host_link_gbs(dev)
    out = {"case": "host", "workload": f"pkm-layer-{rows}-rows-host-table", "rows": rows, "v_dim": D_MODEL, "tokens": N,
           "lookups_per_step": N * HEADS * KNN, "distinct_rows_per_step": distinct, "gacc_capacity": capacity,
           "hot_read_share": round(hot_share, 4), "host_link_gbs": link,
           "host": f"{_cpu_name()}, {threads} threads, {round(_mem_available() / 2**30)} GiB available",
           "steps": args.steps, "warmup": args.warmup, "configs": {}}
    table_gb = rows * D_MODEL * 4
    wanted = args.host_configs.split(",")
    unknown = set(wanted) - {c[0] for c in HOST_CONFIGS}
    if unknown:
        raise ValueError(f"unknown host configurations: {sorted(unknown)}")
    arms = [(label, ours) for label, ours in (("reference", False), ("this_build", True))
            if args.host_arm in ("both", label)]
    for config in HOST_CONFIGS:
        name, optim, gacc, hot = config
        if name not in wanted:
            continue
        need = (0 if gacc else table_gb) + (2 * table_gb if optim == "adam" else 0) + (16 << 30)
        entry = out["configs"][name] = {}
        for label, ours in arms:
            arm = _host_arm(ours)
            if arm is None:
                entry[label] = {"unavailable": "the reference package is not in baseline/_ref"}
                continue
            if _mem_available() < need:
                entry[label] = {"skipped": f"needs {need / 2**30:.0f} GiB of host RAM"}
                continue
            entry[label] = _host_config(arm, ours, config, table, n_keys, xs, gs, reads, capacity, dev,
                                        args.steps, args.warmup)
        ours = entry.get("this_build", {})
        if "ms_per_step" in ours:
            # the host-link roofline of this build's step: the rows' bytes that must cross the link each way
            # (U distinct rows in host RAM per step, rows of 4 * v_dim bytes) over the measured copy bandwidths
            rb = D_MODEL * 4
            if gacc:
                # rows in host RAM per step (HOT rows excluded); those the previous step also read come from the
                # device cache, so only the others cross the link inwards
                cold = hot_cold if hot else plain_cold
                gb_in, gb_out = (cold[0] - cold[1]) * rb / 1e9, cold[0] * rb / 1e9
                rows_in, rows_out = round(1 - cold[1] / cold[0], 3), 1
            else:
                u = statistics.mean(distinct)
                rows_in, rows_out = {"adam": (5, 4), "rowrms": (3, 2)}[name]
                gb_in, gb_out = u * rows_in * rb / 1e9, u * rows_out * rb / 1e9
            serial = (gb_in / link["h2d"] + gb_out / link["d2h"]) * 1e3
            duplex = max(gb_in / link["h2d"], gb_out / link["d2h"]) * 1e3
            ours["host_link"] = {"rows_in_per_row": rows_in, "rows_out_per_row": rows_out, "gb_in": round(gb_in, 2),
                                 "gb_out": round(gb_out, 2), "serial_ms": round(serial, 1),
                                 "duplex_ms": round(duplex, 1), "frac": round(serial / ours["ms_per_step"], 3)}
        if "ms_per_step" in entry.get("reference", {}) and "ms_per_step" in ours:
            entry["speedup"] = round(entry["reference"]["ms_per_step"] / ours["ms_per_step"], 2)
        print(json.dumps({"case": "host", "config": name, **entry}), flush=True)
    return out


# ------------------------------------------------------------------------------------------- inference
def _event_ms(fn, reps):
    """Device time of `reps` calls of fn (CUDA events on the current stream, synchronised on both sides)."""
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e)


@torch.no_grad()
def run_inference(args, local, world=1):
    """The B-16M inference token loop (the metric's "B-16M decode tok/s"): the reference's B-16M
    model (12 layers, d_model 384, 6 attention heads, SwiGLU 1024, vocab 50304, product-key memories in layers 2,
    6 and 10 sharing one 4096^2 = 16,777,216 x 384 fp32 value table, BatchNorm queries, swilu), random-init
    weights, eval mode, bf16 autocast, through smlm_b200.model.Transformer. Measured like the reference's
    inference_benchmark (smlm/train.py:283-315): prefill of 2048 uniform random token ids at batch 1 and 64 (full
    forward, logits of every position), then 256 greedy decode steps from that prefill: decode_b* through
    smlm_b200.decode.GraphDecoder (static KV cache, the whole step one CUDA graph), decode_b*_eager (one GPU only)
    through the reference's loop (growing KV cache, one-token memory layers replaying their own graphs). Plus the
    per-token product-key lookup latency: one memory layer on one token (query projection, fused scoring + top-k
    + softmax, value bag with the swilu product) and, on one GPU, the lookup alone (fused scoring + selection,
    value bag), each as a CUDA-graph replay. On N > 1 GPUs the table is row-sharded over them (peer exchange, the
    swilu product fused into its sum), every rank runs its own prompts (batch b per rank) and the tokens/s are
    whole-job figures (N x b sequences) over the slowest rank's time. All device-timed with CUDA events."""
    from smlm_b200 import kernels as K
    from smlm_b200.decode import GraphDecoder
    from smlm_b200.model import ModelConfig, Transformer
    dev = torch.device("cuda", local)
    prompt, new = 2048, 256
    cfg = ModelConfig(mem_layers=[2, 6, 10], mem_n_keys=args.rows_per_half, mem_share_values=True,
                      mem_value_grad="row_sparse", max_seq_len=prompt + new)
    torch.manual_seed(0)
    group = torch.distributed.group.WORLD if world > 1 else None
    with torch.device(dev):
        model = Transformer(cfg, shard_group=group)
    if world > 1:
        from smlm_b200.sharded import broadcast_replicated
        broadcast_replicated(model, group)
    model.eval()
    model.set_memory_decode_graphs(True)
    rank = torch.distributed.get_rank() if world > 1 else 0
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    res = {"model": "B-16M (12 layers, PKM in layers 2/6/10 sharing one table)" if args.rows_per_half == 4096
           else f"B ({args.rows_per_half ** 2} rows)", "rows": args.rows_per_half ** 2, "prompt_len": prompt,
           "new_tokens": new, "dtype": "bf16 autocast, fp32 value table", "data": "synthetic uniform token ids",
           "gpus": world, "table": "one GPU" if world == 1 else f"row-sharded over {world} GPUs (peer exchange)",
           "batch_is_per_gpu": True}

    def timed(fn, reps):
        return max_over_ranks(_event_ms(fn, reps), world)

    with torch.autocast("cuda", dtype=torch.bfloat16):
        for b in (1, 64):
            ids = torch.randint(0, cfg.vocab_size, (b, prompt), device=dev, generator=gen)
            model(ids)                                                     # warm-up
            reps = 5 if b == 1 else 2
            ms = timed(lambda: model(ids), reps) / reps
            res[f"prefill_b{b}_tok_s"] = round(world * b * prompt / (ms / 1e3), 1)
            res[f"prefill_b{b}_ms"] = round(ms, 3)
            if world == 1:
                for rep in range(2):                                       # rep 0: warm-up (graph capture)
                    caches = [dict() for _ in range(cfg.n_layers)]
                    logits = model(ids, kv_caches=caches, pos0=0)
                    state = {"nxt": logits[:, -1:].argmax(-1), "i": 0}
                    del logits
                    steps = 8 if rep == 0 else new

                    def decode_step():
                        lg = model(state["nxt"], kv_caches=caches, pos0=prompt + state["i"])
                        state["nxt"] = lg[:, -1:].argmax(-1)
                        state["i"] += 1
                    ms = _event_ms(decode_step, steps)
                res[f"decode_b{b}_eager_tok_s"] = round(b * new / (ms / 1e3), 1)
                del caches, state
            dec = GraphDecoder(model, b, max_len=prompt + new)
            dec.prefill(ids)
            dec.step()                                                     # capture
            dec.prefill(ids)
            ms = timed(dec.step, new)
            res[f"decode_b{b}_tok_s"] = round(world * b * new / (ms / 1e3), 1)
            res[f"decode_b{b}_ms_per_step"] = round(ms / new, 4)
            del dec, ids
        # one memory layer, one token: the layer's decode graph
        mem = model.memory_layers()[0]
        x1 = torch.randn(1, cfg.d_model, device=dev, generator=gen)
        for _ in range(3):
            mem(x1)
        res["pkm_layer_us_per_token"] = round(timed(lambda: mem(x1), 200) / 200 * 1e3, 2)
    if world == 1:
        # the lookup alone: fused scoring + top-k + softmax and the value bag of one token, captured once
        q1 = torch.randn(1, mem.heads, mem.k_dim, device=dev, generator=gen).bfloat16()
        keys = mem.keys.detach().bfloat16()
        table = mem.values.weight.detach()

        def lookup():
            _, idx, w = K.score_select(q1, keys, mem.knn)
            return K.bag_infer(idx.view(1, -1), w.view(1, -1), table, out_bf16=True)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                lookup()
        torch.cuda.current_stream(dev).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            lookup()
        for _ in range(3):
            graph.replay()
        res["pkm_lookup_us_per_token"] = round(_event_ms(graph.replay, 200) / 200 * 1e3, 2)
        del graph
    else:
        x = getattr(mem.values.weight, "peer_exchange", None)
        torch.cuda.synchronize(dev)
        for m in model.memory_layers():
            m._graph = None
        if x is not None:
            x.close()
    del model
    return res


# ----------------------------------------------------------------------------------------- CPU reference
REF_PKG = os.path.join(ROOT, "baseline", "_ref")


def _cpu_name():
    try:
        return [ln.split(":", 1)[1].strip() for ln in open("/proc/cpuinfo") if ln.startswith("model name")][0]
    except (OSError, IndexError):
        return "unknown"


def reference_modules():
    """The reference's own modules: its smlm package as vendored, unmodified, into baseline/_ref by
    __graft_entry__.build() (kind "reference"); without it, the restatement under oracle/ (kind "port")."""
    if os.path.isfile(os.path.join(REF_PKG, "smlm", "pkm.py")):
        if REF_PKG not in sys.path:
            sys.path.insert(0, REF_PKG)
        from smlm.pkm import ProductKeyMemory
        from smlm.sparse_values import LazyRowAdam, clip_row_sparse
        return "reference", "the reference's smlm package (baseline/_ref/smlm, unmodified)", \
            (lambda **kw: ProductKeyMemory(impl="torch", **kw)), \
            (lambda params, **kw: LazyRowAdam(params, impl="torch", **kw)), clip_row_sparse
    from oracle import torch_path as TP
    return "port", "the reference's PyTorch path restated in oracle/torch_path.py", \
        (lambda **kw: TP.TorchPKM(canonical=False, **kw)), TP.TorchLazyRowAdam, TP.clip_row_sparse


def cpu_reference(n_keys, N, steps, warmup, threads=None):
    """The reference's PyTorch path on the host cores, one PKM layer step as the GPU arm's (config-1 layer without
    BatchNorm / swilu, fp32: the reference scores in fp32 off CUDA): forward, backward into its RowStore, value
    clipping, its LazyRowAdam (impl="torch": a full-table fused Adam with the unread rows restored) and AdamW on
    the dense parameters. Median of `steps` timed steps after `warmup`."""
    kind, what, PKM, LRA, clip = reference_modules()
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    mem = PKM(d_in=D_MODEL, d_out=D_MODEL, n_keys=n_keys, heads=HEADS, knn=KNN, k_dim=K_DIM, query_norm="none",
              swilu=False, value_grad="row_sparse")
    with torch.no_grad():                                  # config-1 initialisation
        mem.query_proj.weight.normal_(0, 0.02)
        mem.query_proj.bias.zero_()
        mem.keys.normal_(0, (K_DIM // 2) ** -0.5)
        mem.values.weight.normal_(0, D_MODEL ** -0.5)
    table = mem.values.weight
    dense = [p for p in mem.parameters() if p is not table]
    adamw = torch.optim.AdamW(dense, lr=1e-3, betas=(0.9, 0.98), weight_decay=0.0)
    lazy = LRA([table], lr=1e-3, betas=(0.9, 0.98))
    gen = torch.Generator().manual_seed(1)
    xs = [torch.randn(N, D_MODEL, generator=gen) for _ in range(2)]
    gs = [torch.randn(N, D_MODEL, generator=gen) for _ in range(2)]

    def step(i):
        out = mem(xs[i % 2])
        out.backward(gs[i % 2])
        clip([table], 1.0)
        torch.nn.utils.clip_grad_norm_(dense, 1.0)
        adamw.step()
        lazy.step()
        adamw.zero_grad(set_to_none=True)

    for i in range(warmup):
        step(i)
    times = []
    for i in range(steps):
        t0 = time.perf_counter()
        step(i)
        times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    return {"value": round(N / dt, 1), "unit": "tokens/s", "cores": threads, "kind": kind,
            "sample": f"{what} on {_cpu_name()}: one PKM layer step with {n_keys}^2 = {n_keys ** 2} rows x "
                      f"{D_MODEL} (the 16.8M-row table scaled down to fit a bounded CPU run; the reference's "
                      f"full-table Adam makes larger tables slower), {N} tokens per step, median of {steps} timed "
                      f"steps after {warmup} warm-up, {threads} threads",
            "ms_per_step": round(dt * 1e3, 2), "rows": n_keys ** 2, "tokens_per_step": N}


def run_reference_arm(args, world, rank):
    """--impl reference: rank 0 times the reference's CPU path with every host thread on the arm's workload, as a
    bounded sample (a 1M-row table, 4,096 tokens per step), --steps timed steps after --warmup; it also times
    BASELINE config 1 exactly (65,536 rows, 2,048 tokens). Other ranks exit at once without touching a GPU."""
    if rank != 0:
        return None
    base = cpu_reference(args.cpu_rows_per_half, args.cpu_tokens, args.steps, args.warmup)
    c1 = cpu_reference(256, 2048, max(3, min(args.steps, 10)), 2)
    return {"metric": METRIC, "value": base["value"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": base["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "pkm-layer-b16m", "sample": f"pkm-layer-{base['rows']}-rows-cpu-sample",
                       "rows": base["rows"], "tokens_per_step": base["tokens_per_step"], "v_dim": D_MODEL,
                       "heads": HEADS, "knn": KNN, "k_dim": K_DIM,
                       "note": "the B-16M layer step on the host cores, on a bounded sample: see cpu_baseline"},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "config1_cpu": {"rows": c1["rows"], "tokens_per_step": c1["tokens_per_step"], "value": c1["value"],
                            "unit": "tokens/s", "ms_per_step": c1["ms_per_step"], "kind": c1["kind"],
                            "cores": c1["cores"]},
            "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    args = parse()
    if args.case == "scoring":
        run_scoring_case(args)
        return
    if args.case == "configs":
        print(json.dumps({"case": "configs", "steps": args.steps, "warmup": args.warmup,
                          "configs": run_configs(args)}), flush=True)
        return
    if args.case == "engram":
        print(json.dumps(run_engram(args)), flush=True)
        return
    if args.case == "model":
        line = run_model_case(args) if args.model == "b1m" and args.impl == "cuda" else run_model_b16m(args)
        print(json.dumps(line), flush=True)
        return
    if args.case == "host":
        print(json.dumps(run_host(args)), flush=True)
        return
    if args.case == "inference":
        print(json.dumps({"case": "inference", **run_inference(args, 0)}), flush=True)
        return
    if args.impl == "reference":
        # the CPU path needs no process group and no GPU: ranks other than 0 leave at once
        line = run_reference_arm(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup(args)
    line = run_cuda(args, world, rank, local)
    if not args.no_inference:
        import gc
        gc.collect()
        torch.cuda.empty_cache()
        line["inference"] = run_inference(args, local, world)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_reference(args.cpu_rows_per_half, args.cpu_tokens, 3, 1)
        line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
