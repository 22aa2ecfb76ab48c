"""bench.py — the synthetic-encoder throughput of config 2 on 1..8 B200, plus the dominant kernel's
roofline, the reference CPU path timed on this host's cores, and the reference arm.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl e2cuda|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

One step = one pass of the 24-layer synthetic encoder (benchmark config 2: hidden 768, 3 q heads /
1 KV head of 256, FFN 1152, int8 token table [262144][768], dense 768->3072->768, L2) over a batch of
64 sequences x 512 tokens per GPU (weak scaling: every rank embeds its own batch), followed, for
N > 1, by the single NCCL all-gather of the pooled embeddings to every rank.
Inputs are device-resident token ids ("value"); "e2e" drives the same pass through the C ABI's
host-buffer entry point (pinned ids in, embeddings out, copies inside the timed region). Weights are
random-init and seeded, token ids uniform in [2, 262144): there is no checkpoint or dataset.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "encoder embeddings/sec (config-2 synthetic encoder, W8A8 int8 GEMMs)"
UNIT = "embeddings/s"
BATCH, SEQ = 64, 512
CHUNK = BATCH * SEQ


def load_pkg():
    if "e2c_b200" in sys.modules:
        return sys.modules["e2c_b200"]
    pkg = ROOT / "e2.c_b200"
    spec = importlib.util.spec_from_file_location("e2c_b200", pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["e2c_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


# ------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampled every 100 ms (read-only queries). Started before the warm-up; the host marks
    the timed region with mark_start() / mark_end() and the summary covers the samples taken inside
    it, or, when the region is shorter than a few sampling periods, those of warm-up and region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.t0 = self.t1 = None
        self.started = threading.Event()

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            self.started.wait(timeout=5.0)  # the first sample is in before anything is timed
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))
            self.started.set()

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)  # one more sample after the region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        window = "timed region"
        rows = [ln for t, ln in self.lines if self.t0 is not None and self.t0 <= t <= (self.t1 or t)]
        if len(rows) < 3:
            window = "warm-up and timed region (region shorter than 3 sampling periods)"
            rows = [ln for t, ln in self.lines if self.t1 is None or t <= self.t1 + 0.15]
        sm, smax, reasons = [], None, set()
        for ln in rows:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "window": window}


def cpu_info(threads: int) -> dict:
    """The host CPU the baseline ran on: model, ISA flags the reference kernels use, logical CPUs,
    the threads used and their pinning (the process's CPU affinity)."""
    model, flags = None, set()
    try:
        for ln in open("/proc/cpuinfo"):
            if model is None and ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
            if ln.startswith("flags"):
                for f in ln.split(":", 1)[1].split():
                    if f.startswith(("avx512", "amx")) or f in ("avx_vnni", "avx2", "fma"):
                        flags.add(f)
    except OSError:
        pass
    try:
        aff = sorted(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        aff = []
    return {"cpu_model": model, "isa": sorted(flags), "nproc": os.cpu_count(), "threads": threads,
            "pinning": f"process affinity {len(aff)} CPUs ({aff[0]}-{aff[-1]})" if aff else "unknown",
            "pool": "reference thread pool (src/threads.c), one worker per thread, capped at 64"}


# ------------------------------------------------------------------------------------ distributed
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 or n_gpus > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=None)
        return dist, rank, world, local
    return None, 0, 1, 0


def max_over_ranks(dist, value: float, device) -> float:
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------ reference arm
def cpu_reference(seqs: int, seq_len: int, steps: int, warmup: int, weights, rng, budget_s: float | None = None):
    """Times the reference's own CPU int8 path (the e2.c kernels built from source, driven by the
    oracle's encoder composition over the reference thread pool) on `seqs` sequences per step.
    Returns (embeddings/s, info)."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle_ffi as of

    kind = "reference" if of.mux() is not None else "port"
    nthreads = 0
    if kind == "reference":
        nthreads = of.mux().e2refmux_init(str(of.REF_DIR).encode(), 0)
    ids = weights_ids = None
    times = []
    done = 0
    t_start = time.perf_counter()
    for i in range(warmup + steps):
        weights_ids = rng.integers(2, weights.cfg.vocab, size=(seqs, seq_len), dtype=np.int32)
        t0 = time.perf_counter()
        of.encoder_forward(kind, weights, weights_ids)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
            done += seqs
        if budget_s is not None and time.perf_counter() - t_start > budget_s and len(times) >= 1:
            break
    total = sum(times)
    cores = nthreads if kind == "reference" else 1
    info = {"kind": kind, "cores": cores,
            "sample": f"{len(times)} x {seqs} sequences x {seq_len} tokens of the 24-layer encoder "
                      f"({'reference e2.c AVX512-VNNI kernels + thread pool' if kind == 'reference' else 'plain-C port'}), "
                      f"host {os.cpu_count()} logical CPUs"}
    info.update(cpu_info(cores))
    return done / total, info


# ------------------------------------------------------------------------------------ main arm
def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="e2cuda", choices=["e2cuda", "reference"])
    ap.add_argument("--layers", type=int, default=24, help=argparse.SUPPRESS)  # debugging only; headline uses 24
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ablk", type=int, default=0, choices=[0, 128],
                    help="activation block: 0 = per token (the headline), 128 = the reference engine's default recipe")
    ap.add_argument("--kernel", default=None, choices=list(KERNELS),
                    help="run one encoder kernel --steps times at the encoder's shapes (for ncu captures)")
    ap.add_argument("--tokens", type=int, default=BATCH * SEQ, help="tokens for --kernel (a multiple of 512)")
    ap.add_argument("--chunk", type=int, default=CHUNK,
                    help="tokens per device pass (whole sequences); intermediates of a pass stay L2-resident")
    ap.add_argument("--sweep", action="store_true", help="benchmark config 3: the GEMM over M x (K, N)")
    ap.add_argument("--config4", action="store_true",
                    help="benchmark config 4: log-uniform lengths, length-bucketed, LPT-sharded over the GPUs")
    ap.add_argument("--sequences", type=int, default=65536, help="sequences of the config-4 job")
    ap.add_argument("--cpu-subsample", type=int, default=64,
                    help="config 4: time the reference CPU path on every n-th sequence by length (0: skip)")
    ap.add_argument("--config0", action="store_true", help="benchmark config 0: one quantised linear layer")
    ap.add_argument("--config1", action="store_true", help="benchmark config 1: the int8 gated FFN block")
    ap.add_argument("--text-tower", action="store_true",
                    help="benchmark e2.c's own text tower (EmbeddingGemma-2, seeded random-init checkpoint)")
    ap.add_argument("--seq-len", type=int, default=SEQ, help="tokens per sequence for --text-tower")
    args = ap.parse_args()
    if args.kernel:
        return kernel_only(args)
    if args.sweep:
        return gemm_sweep(args)
    if args.config4:
        return config4(args)
    if args.config0:
        return config0(args)
    if args.config1:
        return config1(args)
    if args.text_tower:
        return text_tower(args)

    import torch

    if args.impl == "reference":
        # the reference arm's ranks never communicate (rank 0 times the CPU path, the others exit),
        # so it joins no process group
        dist, rank, world = None, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
    else:
        dist, rank, world, local = dist_setup(args.gpus)
    n = world
    load_pkg()
    import e2c_b200.synthetic as syn

    cfg = syn.EncoderConfig(n_layers=args.layers, max_seq=SEQ)
    config = {"workload": f"config 2: synthetic encoder, {cfg.n_layers} layers, hidden {cfg.hidden}, "
                          f"{cfg.n_heads}q/{cfg.n_kv_heads}kv heads x {cfg.head_dim}, ffn {cfg.ffn}, int8 table "
                          f"[{cfg.vocab}][{cfg.hidden}], head {cfg.hidden}->{cfg.dense_hidden}->{cfg.out_dim}",
              "batch_per_gpu": BATCH, "seq_len": SEQ, "global_batch": BATCH * n,
              "act_scales": "per-token" if not args.ablk else "per-128-block",
              "parallelism": f"dp{n} (batch-sharded, weights replicated, one all-gather)",
              "l2": "inputs larger than L2: each step streams ~0.1 GB of layer weights per pass and ~0.6 GB of ids, "
                    "table rows and activations",
              "tokens_per_pass": args.chunk}

    if args.impl == "reference":
        if rank != 0:
            if dist:
                dist.destroy_process_group()
            return 0
        w = syn.encoder_weights(cfg, ablk=args.ablk or None)
        rng = np.random.default_rng(7)
        seqs = 2
        v, info = cpu_reference(seqs, SEQ, args.steps, args.warmup, w, rng)
        line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": n, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1e3 * seqs / v, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8", "data": "synthetic (seeded random-init weights, uniform token ids)", "config": config,
                "impl": "reference", "cpu_baseline": dict(info, value=v, unit=UNIT),
                "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        if dist:
            dist.destroy_process_group()
        return 0

    e2c = load_pkg()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    w = syn.encoder_weights(cfg, ablk=args.ablk or None)
    desc, keep = syn.fill_desc(w, e2c.Q8W, e2c.EncoderDesc)
    enc = e2c.Encoder(desc, keep, args.chunk)
    rng = np.random.default_rng(1000 + rank)
    ids_host = syn.token_batch(rng, BATCH, SEQ, cfg.vocab)
    ids = torch.from_numpy(ids_host).to(dev)
    out = torch.empty((BATCH, cfg.out_dim), dtype=torch.float32, device=dev)
    gathered = torch.empty((n * BATCH, cfg.out_dim), dtype=torch.float32, device=dev) if dist else None
    stream = torch.cuda.Stream(device=dev)

    def step():
        enc.embed_batch_device(ids, None, out, stream)
        if dist:
            with torch.cuda.stream(stream):
                dist.all_gather_into_tensor(gathered, out)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            for _ in range(max(args.warmup, 3)):
                step()
        e2c.check(stream)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        clk.mark_start()
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                step()
            ev1.record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    e2c.check(stream)
    ms = ev0.elapsed_time(ev1)
    ms = max_over_ranks(dist, ms, dev)
    value = n * BATCH * args.steps / (ms / 1e3)
    _, kernels, _ = enc.stats()
    passes = -(-BATCH // max(args.chunk // SEQ, 1))  # device passes per step (whole sequences per pass)

    # e2e: the host-buffer C-ABI entry point, pinned ids in, embeddings out, copies in the region
    ids_pin = torch.from_numpy(ids_host).pin_memory()
    out_pin = torch.empty((BATCH, cfg.out_dim), dtype=torch.float32).pin_memory()
    for _ in range(2):
        enc.embed_batch_into(ids_pin, None, out_pin)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        enc.embed_batch_into(ids_pin, None, out_pin)
    e2e_ms = (time.perf_counter() - t0) * 1e3
    e2e_ms = max_over_ranks(dist, e2e_ms, dev)
    e2e = n * BATCH * args.steps / (e2e_ms / 1e3)

    # every kernel of a layer in isolation; the roofline object is the dominant one's
    roof, table, small_m = None, None, None
    if rank == 0:
        table = kernel_table(dev, stream) if not args.ablk else None
        roof = dominant_roofline(table) if table else None
        if world == 1 and not args.ablk:
            # the small-activation GEMMs (benchmark config 3 at M = 1 and 16), timed after the pass
            small_m = small_m_table(dev, stream)
    cpu = None
    if world > 1:
        # timed on rank 0 at N = 1 only: with N > 1 the other ranks' NCCL progress threads poll on the
        # same host cores and the sample would measure that contention
        cpu = {"value": None, "unit": UNIT, "note": "the CPU baseline is timed at N=1 only (bench.py --gpus 1)"}
    elif not args.no_cpu_baseline:
        try:
            v, info = cpu_reference(2, SEQ, 3, 1, w, np.random.default_rng(9), budget_s=30.0)
            cpu = dict(info, value=v, unit=UNIT)
        except Exception as ex:  # the baseline is reported, not required
            cpu = {"value": None, "unit": UNIT, "error": str(ex)[:200]}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic (seeded random-init int8 weights, uniform token ids)", "config": config,
                "clocks": clk.summary(),
                "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": int(ids_pin.numel() * 4),
                        "d2h_bytes_per_step": int(out_pin.numel() * 4)},
                "gpu_launches": int(kernels * passes * args.steps), "roofline": roof,
                "kernels": {k: {kk: v[kk] for kk in ("bound", "achieved", "unit", "frac", "avg_ms", "traffic")}
                            for k, v in (table or {}).items()},
                "small_m": small_m,
                "cpu_baseline": cpu}
        print(json.dumps(line))
    enc.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def config4(args) -> int:
    """Benchmark config 4: `--sequences` sequences with lengths floor(exp(U[ln 32, ln 2048])), token ids
    uniform in [2, 262144), bucketed to multiples of 64 tokens, assigned to the ranks by LPT on the
    encoder's cost model, embedded in passes of at most --chunk tokens, and gathered to every rank
    in original order by one all-gather. Ids and masks are on the device before timing; the timed
    region is every rank's passes plus the gather (CUDA events, max over ranks)."""
    import torch

    dist, rank, world, local = dist_setup(args.gpus)
    e2c = load_pkg()
    import e2c_b200.shard as shard
    import e2c_b200.synthetic as syn

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = syn.EncoderConfig(n_layers=args.layers, max_seq=2048)
    w = syn.encoder_weights(cfg)
    desc, keep = syn.fill_desc(w, e2c.Q8W, e2c.EncoderDesc)
    enc = e2c.Encoder(desc, keep, args.chunk)
    rng = np.random.default_rng(44)  # the same job on every rank
    lengths = shard.log_uniform_lengths(rng, args.sequences)
    padded = shard.bucket_length(lengths, 64)
    shares = shard.lpt_assign(shard.sequence_cost(padded, cfg.n_layers), world)
    mine = shares[rank]
    passes = shard.plan_passes(mine, padded, args.chunk)
    tok_rng = np.random.default_rng(45 + rank)
    dev_passes = []
    for ps in passes:
        ids, valid = shard.pack_batch(lambda i: tok_rng.integers(2, cfg.vocab, size=int(lengths[i]), dtype=np.int32),
                                      lengths, ps)
        out = torch.empty((len(ps.seqs), cfg.out_dim), dtype=torch.float32, device=dev)
        dev_passes.append((torch.from_numpy(ids).to(dev), torch.from_numpy(valid).to(dev), out, ps.seqs))
    stream = torch.cuda.Stream(device=dev)
    emb = torch.empty((len(mine), cfg.out_dim), dtype=torch.float32, device=dev)
    pos = {int(i): k for k, i in enumerate(mine)}
    rows = [torch.as_tensor([pos[int(i)] for i in ps_seqs], dtype=torch.int64, device=dev)
            for _, _, _, ps_seqs in dev_passes]

    def run():
        with torch.cuda.stream(stream):
            for (ids, valid, out, _), r in zip(dev_passes, rows):
                enc.embed_batch_device(ids, valid, out, stream)
                emb.index_copy_(0, r, out)
            if dist:
                return shard.gather_embeddings(dist, shares, emb, args.sequences, device=dev)
        return emb

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    mids = []  # per step: this rank's passes done, before the gather
    with ClockSampler(local) as clk:
        for _ in range(2):  # every pass shape runs eagerly once, then is captured as a CUDA graph
            run()
        e2c.check(stream)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        clk.mark_start()
        ev0.record(stream)
        for _ in range(args.steps):
            with torch.cuda.stream(stream):
                st = torch.cuda.Event(enable_timing=True)
                st.record(stream)
                for (ids, valid, out, _), r in zip(dev_passes, rows):
                    enc.embed_batch_device(ids, valid, out, stream)
                    emb.index_copy_(0, r, out)
                m = torch.cuda.Event(enable_timing=True)
                m.record(stream)
                mids.append((st, m))
                if dist:
                    shard.gather_embeddings(dist, shares, emb, args.sequences, device=dev)
        ev1.record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    e2c.check(stream)
    total = ev0.elapsed_time(ev1)
    # this rank's own share of the step (its passes) and the gather's, averaged over the steps
    compute = sum(a.elapsed_time(b) for a, b in mids) / args.steps
    per_rank = torch.tensor([total / args.steps, compute], dtype=torch.float64, device=dev)
    if dist:
        allr = torch.zeros((world, 2), dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(allr, per_rank[None, :])
        per_rank_list = allr.cpu().numpy()
    else:
        per_rank_list = per_rank.cpu().numpy()[None, :]
    ms = float(per_rank_list[:, 0].max())
    cpu = None
    if rank == 0 and world == 1 and args.cpu_subsample > 0:
        cpu = config4_cpu(w, lengths, args.cpu_subsample)
    if rank == 0:
        tokens = int(lengths.sum())
        fin = per_rank_list[:, 1]
        print(json.dumps({"metric": "config-4 embeddings/sec (log-uniform lengths, length-bucketed, LPT-sharded)",
                          "value": args.sequences / (ms / 1e3), "unit": "embeddings/s", "n_gpus": world,
                          "steps": args.steps, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                          "tokens_per_s": tokens / (ms / 1e3), "padded_tokens_per_s": int(padded.sum()) / (ms / 1e3),
                          "dtype": "int8", "data": "synthetic (seeded lengths and token ids, random-init weights)",
                          "config": {"workload": "config 4", "sequences": args.sequences, "tokens": tokens,
                                     "bucket": 64, "tokens_per_pass": args.chunk, "passes_rank0": len(passes)},
                          "per_rank_passes_ms": [round(float(v), 3) for v in fin],
                          "rank_spread": {"min_ms": float(fin.min()), "max_ms": float(fin.max()),
                                          "imbalance": float(fin.max() / fin.mean()) if fin.mean() > 0 else None,
                                          "gather_and_rest_ms": float(ms - fin.max())},
                          "clocks": clk.summary(), "cpu_baseline": cpu}))
    enc.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def config4_cpu(w, lengths: np.ndarray, every: int, budget_s: float = 240.0) -> dict:
    """The reference CPU path on a stratified 1/`every` subsample of the config-4 job (every n-th
    sequence in length order, each at its own length, in a seeded random order), extrapolated to the
    whole job. If the budget runs out first, the part done (a random subset of the subsample) is
    extrapolated instead, and the fraction is stated."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle_ffi as of

    kind = "reference" if of.mux() is not None else "port"
    nthreads = of.mux().e2refmux_init(str(of.REF_DIR).encode(), 0) if kind == "reference" else 1
    order = np.argsort(lengths, kind="stable")
    sub = order[every // 2::every]
    rng = np.random.default_rng(46)
    sub = sub[rng.permutation(len(sub))]
    done_tok, done_seq, t_used = 0, 0, 0.0
    for i in sub:
        n = int(lengths[i])
        ids = rng.integers(2, w.cfg.vocab, size=(1, n), dtype=np.int32)
        t0 = time.perf_counter()
        of.encoder_forward(kind, w, ids)
        t_used += time.perf_counter() - t0
        done_tok += n
        done_seq += 1
        if t_used > budget_s:
            break
    frac = done_seq / len(sub)
    scale = len(lengths) / done_seq
    est_s = t_used * scale
    return dict({"kind": kind, "cores": nthreads, "value": len(lengths) / est_s, "unit": "embeddings/s",
                 "tokens_per_s": done_tok / t_used, "extrapolated_job_s": est_s,
                 "sample": f"{done_seq} of a stratified 1/{every} subsample ({len(sub)} sequences; "
                           f"{frac:.0%} done within the {budget_s:.0f} s budget), each sequence at its own length, "
                           f"extrapolated x{scale:.1f} to the {len(lengths)}-sequence job"}, **cpu_info(nthreads))


def _roof(ops: float, nbytes: float, ms: float) -> dict:
    """Both fractions of a run of `ops` int8 operations over `nbytes` algorithmic bytes in `ms`,
    against the measured peaks (int8 dense = 2 x measured bf16)."""
    p = peaks()
    t = ms / 1e3
    tops, gbs = ops / t / 1e12, nbytes / t / 1e9
    int8_peak = 2.0 * p["bf16_tflops"]
    bound = "tensor" if ops / (int8_peak * 1e12) >= nbytes / (p["hbm_gbs"] * 1e9) else "hbm"
    return {"us": ms * 1e3, "tops": tops, "gbs": gbs, "frac_int8_peak": tops / int8_peak,
            "frac_hbm": gbs / p["hbm_gbs"], "bound": bound,
            "frac_of_roofline": (tops / int8_peak) if bound == "tensor" else (gbs / p["hbm_gbs"]),
            "peak_src": f"{p['src']}: HBM {p['hbm_gbs']} GB/s, int8 2 x {p['bf16_tflops']} TFLOP/s"}


def _best_cpu(fn, warmup: int = 2, reps: int = 5, budget_s: float = 20.0) -> float:
    """Best wall time (s) of `fn` after warm-ups (the reference's own rule, PERFORMANCE.md:19-24)."""
    for _ in range(warmup):
        fn()
    best, t_end = math.inf, time.perf_counter() + budget_s
    for i in range(reps):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
        if time.perf_counter() > t_end and i >= 1:
            break
    return best


def config0(args) -> int:
    """Benchmark config 0: y = int8 GEMM(quantise(X)) for X [512][768] N(0,1) with four outlier
    channels x20 and W [1152][768] N(0,0.02) quantised per row by the reference's own weight
    quantiser. Device: the quantiser + GEMM kernels over resident X (L2 flushed before every step);
    e2e: the reference-signature host drop-ins (e2cuda_i8_quantize_host then e2cuda_i8_gemm_host,
    host buffers, copies inside). Beside them the reference's quantise + N-split GEMM region
    (e2ref_linear over its pool) on the host cores."""
    import ctypes as C

    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import oracle_ffi as of

    e2c = load_pkg()
    import e2c_b200.synthetic as syn

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    M, K, N = 512, 768, 1152
    rng = np.random.default_rng(0xE2C0DE + 0)
    x = syn.activations(rng, M, K)
    wf = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    ref = of.ref(K)
    wq = of.Weight(wf, K, lib=ref) if ref is not None else of.Weight(wf, K)
    W = e2c.Weight(q8w=C.cast(C.byref(wq.q), C.POINTER(e2c.Q8W)).contents)
    xd = torch.from_numpy(x).to(dev)
    q = torch.empty((M, K), dtype=torch.int8, device=dev)
    qs = torch.empty((M, 1), dtype=torch.float32, device=dev)
    y = torch.empty((M, N), dtype=torch.float32, device=dev)
    lib = e2c.lib()
    ep = e2c.Epilogue()

    def run():
        e2c._ok(lib.e2cuda_quantize_rows(xd.data_ptr(), q.data_ptr(), qs.data_ptr(), M, K, K, -math.inf, math.inf,
                                         stream.cuda_stream), "quantize")
        e2c._ok(lib.e2cuda_i8_gemm(C.byref(W.w8), q.data_ptr(), qs.data_ptr(), M, K, 0, N, C.byref(ep), y.data_ptr(),
                                   N, stream.cuda_stream), "gemm")

    ms = timed_launches(run, stream, max(args.warmup, 3), args.steps)
    e2c.check(stream)
    ops = 2.0 * M * N * K
    nbytes = 4 * M * K + N * K + 4 * N + 4 * M * N  # x in, W + scales, y out (q stays on chip / in L2)
    # e2e through the reference-signature host drop-ins
    lib.e2cuda_set_act_block(K)
    qa_h = np.empty((M, K), np.int8)
    as_h = np.empty((M, 1), np.float32)
    y_h = np.empty((M, N), np.float32)

    def host_call():
        lib.e2cuda_i8_quantize_host(qa_h.ctypes.data_as(e2c.i8p), as_h.ctypes.data_as(e2c.f32p),
                                    x.ctypes.data_as(e2c.f32p), M, K, -math.inf, math.inf)
        lib.e2cuda_i8_gemm_host(y_h.ctypes.data_as(e2c.f32p), qa_h.ctypes.data_as(e2c.i8p), as_h.ctypes.data_as(e2c.f32p),
                                C.cast(C.byref(wq.q), C.POINTER(e2c.Q8W)), M, N, 0, N)

    for _ in range(3):
        host_call()
    if e2c.last_error():
        raise RuntimeError(e2c.last_error())
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_call()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    cpu = None
    if ref is not None:
        qa_c = np.empty((M, K), np.int8)
        as_c = np.empty((M, 1), np.float32)
        y_c = np.empty((M, N), np.float32)
        nthreads = ref.e2ref_init(0)
        t = _best_cpu(lambda: ref.e2ref_linear(x.ctypes.data_as(of.f32p), M, K, C.byref(wq.q), qa_c.ctypes.data_as(of.i8p),
                                               as_c.ctypes.data_as(of.f32p), y_c.ctypes.data_as(of.f32p)))
        cpu = dict(_roof(ops, nbytes, t * 1e3), kind="reference", cores=nthreads,
                   sample="quantise + N-split int8 GEMM region of e2.c (e2_quantize_blocks_avx512 + e2_i8_gemm_avx512, "
                          "E2_I8_BLOCK=768) over its pool, best of 5 after 2 warm-ups", **cpu_info(nthreads))
    print(json.dumps({"metric": "config-0 quantised linear layer time", "value": ms * 1e3, "unit": "us",
                      "higher_is_better": False, "steps": args.steps, "dtype": "int8",
                      "data": "synthetic (seeded, benchmark config 0)",
                      "config": {"workload": "config 0: quantise X [512][768] + W8A8 GEMM -> fp32 [512][1152], per-row scales",
                                 "l2": "flushed before every step", "kernels_per_step": 2},
                      "roofline": _roof(ops, nbytes, ms), "algorithmic_bytes": nbytes, "ops": ops,
                      "e2e": {"value": e2e_ms * 1e3, "unit": "us", "api": "e2cuda_i8_quantize_host + e2cuda_i8_gemm_host",
                              "h2d_bytes_per_step": 4 * M * K + M * K + 4 * M, "d2h_bytes_per_step": M * K + 4 * M + 4 * M * N},
                      "cpu_baseline": cpu}))
    return 0


def config1(args) -> int:
    """Benchmark config 1: the int8 gated FFN block at M = 4096 tokens (RMSNorm -> quantise -> gate|up
    768->2x1152 -> GELU-tanh(gate)*up -> quantise -> down 1152->768 + residual) through
    e2cuda_ffn_forward (3 kernels). Device time over resident x (L2 flushed before every step); e2e
    with pinned host x / y and the copies inside; beside them the reference's own kernels running the
    same block over its pool on the host cores."""
    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import oracle_ffi as of

    e2c = load_pkg()
    import e2c_b200.synthetic as syn

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    rng = np.random.default_rng(0xE2C0DE + 1)
    M, D, I = 4096, 768, 1152
    x = rng.standard_normal((M, D), dtype=np.float32)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    wg, wu = syn.packed_weight(rng, I, D, 0.02, D), syn.packed_weight(rng, I, D, 0.02, D)
    wd = syn.packed_weight(rng, D, I, 0.02, I)
    qs = [e2c.Q8W() for _ in range(3)]
    for qq, ww in zip(qs, (wg, wu, wd)):
        ww.fill(qq)
    ffn = e2c.FFN(qs[0], qs[1], qs[2], g, 1e-6, M)
    xd = torch.from_numpy(x).to(dev)
    yd = torch.empty_like(xd)
    ms = timed_launches(lambda: ffn.forward(xd, yd, stream), stream, max(args.warmup, 3), args.steps)
    e2c.check(stream)
    ops = 2.0 * M * (D * 2 * I + I * D)
    nbytes = 4 * M * D + (2 * I * D + D * I) + 4 * (2 * I + D) + 4 * M * D + 4 * D  # x in, weights, y out, gamma
    x_pin = torch.from_numpy(x).pin_memory()
    y_pin = torch.empty((M, D), dtype=torch.float32).pin_memory()

    def e2e_step():
        with torch.cuda.stream(stream):
            xd.copy_(x_pin, non_blocking=True)
            ffn.forward(xd, yd, stream)
            y_pin.copy_(yd, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    cpu = None
    if of.mux() is not None:
        nthreads = of.mux().e2refmux_init(str(of.REF_DIR).encode(), 0)
        t = _best_cpu(lambda: of.ffn_block("reference", x, g, 1e-6, wg, wu, wd, ablk=0))
        cpu = dict(_roof(ops, nbytes, t * 1e3), kind="reference", cores=nthreads,
                   sample="the same block on e2.c's own kernels (per-row builds) over its pool, best of 5 after 2 warm-ups",
                   **cpu_info(nthreads))
    print(json.dumps({"metric": "config-1 int8 FFN block time", "value": ms * 1e3, "unit": "us",
                      "higher_is_better": False, "steps": args.steps, "dtype": "int8",
                      "data": "synthetic (seeded, benchmark config 1)",
                      "config": {"workload": "config 1: FFN block, M=4096, D=768, I=1152, per-token scales",
                                 "l2": "flushed before every step", "kernels_per_step": 3},
                      "roofline": _roof(ops, nbytes, ms), "algorithmic_bytes": nbytes, "ops": ops,
                      "e2e": {"value": e2e_ms * 1e3, "unit": "us", "api": "e2cuda_ffn_forward, pinned host x/y",
                              "h2d_bytes_per_step": 4 * M * D, "d2h_bytes_per_step": 4 * M * D},
                      "cpu_baseline": cpu}))
    return 0


def text_pass_work(B: int, S: int, cfg) -> list:
    """(kernel, int8 ops, bf16 flops, algorithmic bytes) of every launch of one text-tower pass over
    B sequences of S tokens (activations per 128-block; the PLE gate, the PLE projection of the
    embeddings, q|k|v on the layers with heads of 512 and embed_proj write fp32; gate|up writes h
    quantised per 128-block, q|k|v on the layers with heads of 256 bf16 Q, K and V^T, and o_proj,
    down and the PLE projection the residual and the next int8 rows)."""
    M, D, I, P, L, H, DO = B * S, cfg.hidden, cfg.intermediate, cfg.ple_dim, cfg.n_layers, cfg.n_heads, cfg.out_dim

    def gemm(name, K, N):
        return (name, 2.0 * M * K * N, 0.0, M * K + 4 * M * K / 128 + N * K + 4 * N + 4 * M * N)

    def gemm_norm(name, K):  # the residual norms in the epilogue: res read and written, int8 rows + scales
        return (name, 2.0 * M * K * D, 0.0, M * K + 4 * M * K / 128 + D * K + 12 * D + 8 * M * D + M * D + 4 * M * D / 128)

    w = [("embed", 0, 0, 4 * M + 2 * M * D + 4 * M * D + 2 * (M * D + 4 * M * D / 128)), gemm("ple_proj_model", D, L * P)]
    for l in range(L):
        hd, kv, qd = cfg.head_dim(l), cfg.n_kv(l), cfg.q_dim(l)
        nqkv = qd + 2 * kv * hd
        keys = S if cfg.full(l) else min(S, 2 * cfg.window + 1)
        if hd == 256:  # the q|k|v finish in the GEMM's epilogue: bf16 Q, K, V^T written once
            w += [("qkv_finish", 2.0 * M * D * nqkv, 0.0, M * D + 4 * M * D / 128 + nqkv * D + 4 * nqkv + 2 * M * nqkv)]
        else:
            w += [gemm("qkv", D, nqkv), ("qkv_post", 0, 0, 4 * M * nqkv + 2 * M * nqkv)]
        w += [("attention", 0, 4.0 * M * keys * hd * H, 2 * M * nqkv + 4 * M * qd),
              ("quantize_ctx", 0, 0, 4 * M * qd + M * qd + 4 * M * qd / 128), gemm_norm("o_proj_norm", qd),
              ("gate_up_gelu_quant", 2.0 * M * D * 2 * I, 0.0,
               M * D + 4 * M * D / 128 + 2 * I * D + 8 * I + M * I + 4 * M * I / 128), gemm_norm("down_norm", I),
              gemm("ple_gate", D, P), ("ple_gate_quant", 0, 0, 8 * M * P + M * P + 4 * M * P / 128),
              gemm_norm("ple_proj_norm", P)]
    w += [gemm("embed_proj", D, DO), ("meanpool", 0, 0, 4 * M * DO), ("l2norm", 0, 0, 8 * B * DO)]
    return w


def text_tower(args) -> int:
    """e2.c's own text tower (EmbeddingGemma-2: hidden 512, 24 layers with per-layer embeddings,
    sliding-window and full attention, embed_proj to 768) on a seeded random-init checkpoint: B x S
    tokens per step through e2cuda_text_embed_batch_device (ids resident), e2e through
    e2cuda_text_embed_batch (pinned host ids and embeddings), a pass roofline (the sum over its
    launches of max(ops / measured peak, bytes / measured HBM)), and beside them e2.c's own engine on
    the host cores running the same checkpoint written as model.safetensors (a bounded sample)."""
    import tempfile

    import torch

    e2c = load_pkg()
    import e2c_b200.text_model as tm

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    cfg = tm.TextConfig()
    B, S = BATCH, args.seq_len
    tensors = tm.random_tensors(cfg)
    w = tm.TextWeights(tensors, cfg)
    tower = e2c.TextTower(w.desc(), B * S, keepalive=w)
    ids_host = tm.token_ids(np.random.default_rng(1000), B, S, cfg.vocab)
    ids = torch.from_numpy(ids_host).to(dev)
    out = torch.empty((B, cfg.out_dim), dtype=torch.float32, device=dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        for _ in range(max(args.warmup, 3)):
            tower.embed_batch_device(ids, None, out, stream)
        e2c.check(stream)
        torch.cuda.synchronize()
        clk.mark_start()
        ev0.record(stream)
        for _ in range(args.steps):
            tower.embed_batch_device(ids, None, out, stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    e2c.check(stream)
    ms = ev0.elapsed_time(ev1) / args.steps
    _, kernels, _ = tower.stats()
    ids_pin = torch.from_numpy(ids_host).pin_memory()
    out_pin = torch.empty((B, cfg.out_dim), dtype=torch.float32).pin_memory()
    for _ in range(2):
        tower.embed_batch_into(ids_pin, None, out_pin)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tower.embed_batch_into(ids_pin, None, out_pin)
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    p = peaks()
    work = text_pass_work(B, S, cfg)
    int8_peak, bf16_peak = 2.0 * p["bf16_tflops"] * 1e12, p["bf16_tflops"] * 1e12
    lb = sum(max(o / int8_peak, f / bf16_peak, b / (p["hbm_gbs"] * 1e9)) for _, o, f, b in work) * 1e3
    ops, flops, nbytes = (sum(x[i] for x in work) for i in (1, 2, 3))
    by_kind = {}
    for name, o, f, b in work:
        by_kind[name] = by_kind.get(name, 0.0) + max(o / int8_peak, f / bf16_peak, b / (p["hbm_gbs"] * 1e9)) * 1e3
    cpu = None
    if not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT))
        from oracle import oracle_ffi as of

        try:
            with tempfile.TemporaryDirectory() as td:
                tm.write_safetensors(Path(td) / "model.safetensors", tensors)
                ref = of.RefText()
                ref.load(td, Path(td) / "text.e8cq")
                seqs = max(1, 2048 // S)  # e2.c's own forward chunk: E2_MAX_SEQ tokens
                sample = ids_host[:seqs]
                t = _best_cpu(lambda: ref.embed_batch(sample), warmup=1, reps=3, budget_s=30.0)
                nthreads = ref.threads()
                cpu = {"value": seqs / t, "unit": "embeddings/s", "kind": "reference", "cores": nthreads,
                       "sample": f"{seqs} x {S} tokens of the same ids through e2.c's own e2_text_embed_batch "
                                 f"(its default int8 attention from 128 keys), best of 3 after 1 warm-up",
                       **cpu_info(nthreads)}
                ref.free()
        except Exception as ex:  # the baseline is reported, not required
            cpu = {"value": None, "unit": "embeddings/s", "error": str(ex)[:200]}
    print(json.dumps({
        "metric": "e2.c text tower throughput", "value": B / (ms / 1e3), "unit": "embeddings/s",
        "tokens_per_s": B * S / (ms / 1e3), "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms, "higher_is_better": True, "dtype": "int8 GEMMs, bf16 attention",
        "data": "synthetic (seeded random-init EmbeddingGemma-2 text tower checkpoint, uniform token ids)",
        "config": {"workload": f"e2.c text tower: {cfg.n_layers} layers, hidden {cfg.hidden}, ffn {cfg.intermediate}, "
                               f"PLE {cfg.n_layers}x{cfg.ple_dim}, 4 heads (256/2kv sliding 512, 512/1kv full), "
                               f"bf16 table [{cfg.vocab}][{cfg.hidden}], embed_proj {cfg.hidden}->{cfg.out_dim}",
                   "batch": B, "seq_len": S, "act_scales": "per-128-block (e2.c's default build)",
                   "l2": "each pass streams ~2 GB of activations (the PLE buffer alone 1.6 GB)"},
        "clocks": clk.summary(),
        "e2e": {"value": B / (e2e_ms / 1e3), "unit": "embeddings/s", "api": "e2cuda_text_embed_batch, pinned host buffers",
                "h2d_bytes_per_step": int(ids_pin.numel() * 4), "d2h_bytes_per_step": int(out_pin.numel() * 4)},
        "gpu_launches": int(kernels * args.steps),
        "pass_roofline": {"lower_bound_ms": lb, "frac": lb / ms, "int8_tops": ops / (ms / 1e3) / 1e12,
                          "bf16_tflops": flops / (ms / 1e3) / 1e12, "algorithmic_gb": nbytes / 1e9,
                          "lower_bound_ms_by_kernel": {k: round(v, 4) for k, v in by_kind.items()},
                          "peak_src": p["src"]},
        "cpu_baseline": cpu}))
    tower.close()
    return 0


# One layer's kernels at the encoder's shape (M = 64 x 512 tokens, hidden 768, FFN 1152, 3 q heads and
# one KV head of 256), the per-launch algorithmic work each is measured against, and the launches of
# each per layer. Weights are quantised N(0, 0.02), activations per-token quantised N(0, 1).
KERNELS = ("gate_up", "gate_up_q", "qkv", "o_proj", "down", "o_proj_norm", "down_norm", "attention", "quantize",
           "quantize_ctx", "norm_add", "o_proj_pb", "down_pb", "gate_up_pb", "gate_up_q_pb", "qkv_pb", "attention_vision",
           "gemm_small")
# gemm_small: the config-3 GEMM (K, N) = (2048, 8192) at M = --tokens rows (1..256) on the
# weight-streaming kernel itself (e2c_gemm_stream), per-token scales, fp32 output
# attention_vision: the vision tower's attention (e2.c src/vision.c:540-571), 2520 patches per image,
# 12 heads of 64 with their own K and V, scale 1; M tokens = M // 2520 images
# *_pb: the same GEMMs with per-128-block activation scales (the reference engine's own recipe);
# gate_up_pb writes g|u in fp32, gate_up_q_pb applies GELU-gate and h's per-block quantiser, qkv_pb
# finishes the heads (RMSNorm, RoPE from position-major tables, bf16 Q, K, V^T)
# the kernels an encoder layer runs (hidden 768, FFN 1152, per-token scales): the residual norms fused
# into o_proj and down and h's quantiser into gate|up, or with E2C_FUSED_NORM=0 / E2C_FUSED_GELU=0
# the row kernels after them
LAYER_KERNELS = ("gate_up_q", "qkv", "o_proj_norm", "down_norm", "attention", "quantize_ctx")
if os.environ.get("E2C_FUSED_NORM") == "0":
    LAYER_KERNELS = tuple(k for k in LAYER_KERNELS if k not in ("o_proj_norm", "down_norm")) + ("o_proj", "down", "norm_add")
if os.environ.get("E2C_FUSED_GELU") == "0":
    LAYER_KERNELS = tuple(k for k in LAYER_KERNELS if k != "gate_up_q") + ("gate_up", "quantize")


GEMM_KERNELS = ("gate_up", "gate_up_q", "qkv", "o_proj", "down", "o_proj_norm", "down_norm", "o_proj_pb", "down_pb",
                "gate_up_pb", "gate_up_q_pb", "qkv_pb")


def kernel_work(name: str, M: int) -> dict:
    D, I, H, Dh = 768, 1152, 3, 256
    if name in GEMM_KERNELS:
        N, K = {"gate_up": (2 * I, D), "gate_up_q": (2 * I, D), "qkv": ((H + 2) * Dh, D), "o_proj": (D, D),
                "down": (D, I), "o_proj_norm": (D, D), "down_norm": (D, I), "o_proj_pb": (D, D), "down_pb": (D, I),
                "gate_up_pb": (2 * I, D), "gate_up_q_pb": (2 * I, D), "qkv_pb": ((H + 2) * Dh, D)}[name]
        # the fused norm epilogue reads and writes the fp32 residual and writes int8 rows + scales;
        # the fused GELU-quantise epilogue writes int8 h + scales
        out_bytes = {"gate_up": 4 * M * I, "gate_up_q": M * I + 4 * M, "qkv": 2 * M * N, "o_proj": 4 * M * D,
                     "down": 4 * M * D, "o_proj_norm": 8 * M * D + M * D + 4 * M,
                     "down_norm": 8 * M * D + M * D + 4 * M, "o_proj_pb": 4 * M * D, "down_pb": 4 * M * D,
                     "gate_up_pb": 8 * M * I, "gate_up_q_pb": M * I + 4 * M * (I // 128), "qkv_pb": 2 * M * N}[name]
        a_scales = 4 * M * (K // 128) if name.endswith("_pb") else 4 * M
        return {"ops": 2.0 * M * N * K, "bytes": M * K + a_scales + N * K + 4 * N + out_bytes, "per_layer": 1}
    if name == "attention":
        return {"ops": 4.0 * M * SEQ * Dh * H, "bytes": M * (H + 2) * Dh * 2 + 4 * M * H * Dh, "per_layer": 1}
    if name == "gemm_small":
        K, N = 2048, 8192
        return {"ops": 2.0 * M * N * K, "bytes": M * K + 4 * M + N * K + 4 * N + 4 * M * N, "per_layer": 1}
    if name == "attention_vision":
        P, Hv, Dv = 2520, 12, 64
        Mv = max(1, M // P) * P
        return {"ops": 4.0 * Mv * P * Dv * Hv, "bytes": Mv * 3 * Hv * Dv * 2 + 4 * Mv * Hv * Dv, "per_layer": 1}
    if name in ("quantize", "quantize_ctx"):
        K = I if name == "quantize" else D
        return {"ops": 0.0, "bytes": M * (4 * K + K + 4), "per_layer": 1}
    return {"ops": 0.0, "bytes": M * (3 * 4 * D + D + 4), "per_layer": 2}  # norm_add


def kernel_runner(name: str, M: int, dev, stream):
    """A closure launching one encoder kernel at token count M (multiple of 512) on `stream`, plus the
    buffers it keeps alive."""
    import ctypes as C

    import torch

    e2c = load_pkg()
    import e2c_b200.synthetic as syn

    D, I, Dh, H = 768, 1152, 256, 3
    g = torch.Generator(device=dev).manual_seed(5)
    rng = np.random.default_rng(5)

    def qin(K):
        return e2c.quantize_rows(torch.randn((M, K), device=dev, generator=g), K)

    keep = []
    if name in GEMM_KERNELS:
        N, K = {"gate_up": (2 * I, D), "gate_up_q": (2 * I, D), "qkv": ((H + 2) * Dh, D), "o_proj": (D, D),
                "down": (D, I), "o_proj_norm": (D, D), "down_norm": (D, I), "o_proj_pb": (D, D), "down_pb": (D, I),
                "gate_up_pb": (2 * I, D), "gate_up_q_pb": (2 * I, D), "qkv_pb": ((H + 2) * Dh, D)}[name]
        wq, ws = syn.quantize_weight_rows((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        W = e2c.Weight(w=wq, scale=ws)
        pb = name.endswith("_pb")
        qa, qs = e2c.quantize_rows(torch.randn((M, K), device=dev, generator=g), 128) if pb else qin(K)
        a = e2c.gemm_args(W, qa, qs, M)
        if pb:
            a.ablk = 128
        keep = [W, qa, qs]
        if name == "gate_up":
            y = torch.empty((M, I), dtype=torch.float32, device=dev)
            a.epi, a.y, a.ldy = e2c.EPI_GELU, y.data_ptr(), I
            keep.append(y)
        elif name in ("gate_up_q", "gate_up_q_pb"):
            q8 = torch.empty((M, I), dtype=torch.int8, device=dev)
            q8s = torch.empty((M, I // 128 if pb else 1), dtype=torch.float32, device=dev)
            a.epi, a.q8, a.ldq, a.q8_scale = e2c.EPI_GELUQ, q8.data_ptr(), I, q8s.data_ptr()
            keep += [q8, q8s]
        elif name == "gate_up_pb":
            y = torch.empty((M, 2 * I), dtype=torch.float32, device=dev)
            a.epi, a.y, a.ldy = e2c.EPI_F32, y.data_ptr(), 2 * I
            keep.append(y)
        elif name in ("down", "o_proj", "down_pb", "o_proj_pb"):
            y = torch.empty((M, D), dtype=torch.float32, device=dev)
            a.epi, a.y, a.ldy = e2c.EPI_F32, y.data_ptr(), D
            keep.append(y)
        elif name in ("down_norm", "o_proj_norm"):
            res = torch.randn((M, D), device=dev, generator=g)
            g1 = torch.ones(D, device=dev)
            q8 = torch.empty((M, D), dtype=torch.int8, device=dev)
            q8s = torch.empty((M,), dtype=torch.float32, device=dev)
            keep += [res, g1, q8, q8s]
            a.epi, a.eps, a.res, a.ldres = e2c.EPI_NORMADD, 1e-6, res.data_ptr(), D
            a.norm_g1 = a.norm_g2 = g1.data_ptr()
            a.q8, a.ldq, a.q8_scale = q8.data_ptr(), D, q8s.data_ptr()
        else:
            Q = torch.empty((M, H * Dh), dtype=torch.bfloat16, device=dev)
            Kt = torch.empty((M, Dh), dtype=torch.bfloat16, device=dev)
            Vt = torch.empty((M // SEQ, Dh, SEQ), dtype=torch.bfloat16, device=dev)
            gam = torch.ones(Dh, device=dev)
            # RoPE tables: pair-major [Dh/2][SEQ] for the per-token epilogue, position-major
            # [SEQ][Dh/2] for the per-block one (the same size)
            cs = torch.rand((Dh // 2, SEQ), device=dev)
            keep += [Q, Kt, Vt, gam, cs]
            a.epi = e2c.EPI_QKVPB if pb else e2c.EPI_QKV
            a.nq, a.q_out, a.k_out, a.vt_out, a.ldvt, a.seq_len = H, Q.data_ptr(), Kt.data_ptr(), Vt.data_ptr(), SEQ, SEQ
            a.q_gamma = a.k_gamma = gam.data_ptr()
            a.rope_cos = a.rope_sin = cs.data_ptr()
            a.ldrope = Dh // 2 if pb else SEQ
            a.eps = 1e-6
        return (lambda: e2c.gemm_raw(a, stream)), keep
    if name == "attention":
        B = M // SEQ
        q = torch.randn((M, H * Dh), device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn((M, Dh), device=dev, generator=g).to(torch.bfloat16)
        vt = torch.randn((B, Dh, SEQ), device=dev, generator=g).to(torch.bfloat16)
        return (lambda: e2c.attention(q, k, vt, None, B, SEQ, H, 1.0 / 16, stream)), [q, k, vt]
    if name == "gemm_small":
        K, N = 2048, 8192
        lib = e2c.lib()
        lib.e2c_gemm_ws_bytes.argtypes = [C.c_int]
        lib.e2c_gemm_ws_bytes.restype = C.c_size_t
        lib.e2cu_status.restype = C.c_void_p
        wq, ws_ = syn.quantize_weight_rows((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        W = e2c.Weight(w=wq, scale=ws_)
        qa, qs = qin(K)
        y = torch.empty((M, N), dtype=torch.float32, device=dev)
        wsb = lib.e2c_gemm_ws_bytes(M)
        wsp = torch.zeros(max(wsb // 4, 1) + 32, dtype=torch.int32, device=dev)
        a = e2c.gemm_args(W, qa, qs, M)
        a.epi, a.y, a.ldy = e2c.EPI_F32, y.data_ptr(), N
        a.status = lib.e2cu_status()
        a.ws, a.ws_bytes = wsp.data_ptr(), wsb
        lib.e2c_gemm_stream.argtypes = [C.POINTER(e2c.GemmArgs), C.c_void_p]
        lib.e2c_gemm_stream.restype = C.c_int
        run = lambda: e2c._ok(lib.e2c_gemm_stream(C.byref(a), e2c._stream(stream)), "gemm_stream")
        return run, [W, qa, qs, y, wsp, a]
    if name == "attention_vision":
        P, Hv, Dv = 2520, 12, 64
        B = max(1, M // P)
        q = torch.randn((B * P, Hv * Dv), device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn((B * P, Hv * Dv), device=dev, generator=g).to(torch.bfloat16)
        vt = torch.randn((B, Hv * Dv, P), device=dev, generator=g).to(torch.bfloat16)
        return (lambda: e2c.attention_gqa(q, k, vt, None, B, P, Hv, Hv, Dv, 1.0, stream)), [q, k, vt]
    if name in ("quantize", "quantize_ctx"):
        K = I if name == "quantize" else D
        x = torch.randn((M, K), device=dev, generator=g)
        q = torch.empty((M, K), dtype=torch.int8, device=dev)
        s_ = torch.empty((M, 1), dtype=torch.float32, device=dev)
        lib = e2c.lib()
        return (lambda: e2c._ok(lib.e2cuda_quantize_rows(x.data_ptr(), q.data_ptr(), s_.data_ptr(), M, K, K,
                                                        -math.inf, math.inf, e2c._stream(stream)), "quantize")), [x, q, s_]
    # norm_add: x = rmsnorm(t) * g1 + res; res = x; q = quantise(rmsnorm(x) * g2), per token
    lib = e2c.lib()
    fn = lib.e2c_norm_add_norm_quant
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p] * 5 + [C.c_float, C.c_void_p, C.c_void_p] + [C.c_int] * 3 + [C.c_void_p]
    t = torch.randn((M, D), device=dev, generator=g)
    res = torch.randn((M, D), device=dev, generator=g)
    g1 = torch.ones(D, device=dev)
    g2 = torch.ones(D, device=dev)
    q = torch.empty((M, D), dtype=torch.int8, device=dev)
    s_ = torch.empty((M, 1), dtype=torch.float32, device=dev)
    run = lambda: e2c._ok(fn(t.data_ptr(), res.data_ptr(), g1.data_ptr(), g2.data_ptr(), None, 1e-6, q.data_ptr(),
                             s_.data_ptr(), M, D, D, e2c._stream(stream)), "norm_add_norm_quant")
    return run, [t, res, g1, g2, q, s_]


def kernel_table(dev, stream, M: int = BATCH * SEQ, steps: int = 10) -> dict:
    """CUDA-event time of every encoder kernel at the encoder's shape (L2 flushed before each launch)
    with its roofline fraction against the measured peaks."""
    e2c = load_pkg()
    traffic = {}
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text())
    table = {}
    for name in LAYER_KERNELS:
        run, keep = kernel_runner(name, M, dev, stream)
        ms = timed_launches(run, stream, 3, steps)
        e2c.check(stream)
        table[name] = dict(binding_roofline(name, M, ms), traffic=traffic.get(name))
        del run, keep
    return table


def binding_roofline(name: str, M: int, ms: float) -> dict:
    """Kernel `name` at M tokens taking `ms`: the binding roofline (whichever of the tensor-core time
    and the HBM time at the measured peaks is longer) and the fraction of it achieved."""
    p = peaks()
    wk = kernel_work(name, M)
    tpeak, hbm = (p["bf16_tflops"] if name.startswith("attention") else 2.0 * p["bf16_tflops"]), p["hbm_gbs"]
    bound = "tensor" if wk["ops"] / (tpeak * 1e12) >= wk["bytes"] / (hbm * 1e9) else "hbm"
    if bound == "tensor":
        peak, achieved, unit = tpeak, wk["ops"] / (ms / 1e3) / 1e12, "TFLOP/s"
    else:
        peak, achieved, unit = hbm, wk["bytes"] / (ms / 1e3) / 1e9, "GB/s"
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak, "avg_ms": ms,
            "launches_per_layer": wk["per_layer"], "algorithmic_bytes": wk["bytes"]}


def dominant_roofline(table: dict) -> dict:
    """The roofline of the kernel with the largest share of a layer's time (time x launches per layer)."""
    name = max(table, key=lambda k: table[k]["avg_ms"] * table[k]["launches_per_layer"])
    p = peaks()
    r = dict(table[name])
    r["kernel"] = name
    if r["bound"] == "hbm":
        r["peak_src"] = f"{p['src']} HBM copy {p['hbm_gbs']} GB/s"
    elif name == "attention":
        r["peak_src"] = f"{p['src']} bf16 {p['bf16_tflops']} TFLOP/s"
    else:
        r["peak_src"] = f"2 x {p['src']} bf16 {p['bf16_tflops']} TFLOP/s (dense int8 = 2 x dense bf16; int8 ops counted as FLOP)"
    return r


def kernel_only(args) -> int:
    """One encoder kernel in isolation (the ncu capture target): prints its CUDA-event average."""
    import torch

    e2c = load_pkg()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    run, keep = kernel_runner(args.kernel, args.tokens, dev, stream)
    avg_ms = timed_launches(run, stream, args.warmup, args.steps)
    e2c.check(stream)
    r = binding_roofline(args.kernel, args.tokens, avg_ms)
    print(json.dumps({"kernel": args.kernel, "tokens": args.tokens, "avg_ms": avg_ms, "l2": "flushed between launches",
                      "bound": r["bound"], "achieved": r["achieved"], "unit": r["unit"], "frac": r["frac"]}))
    return 0


def timed_launches(run, stream, warmup: int, steps: int) -> float:
    """Average CUDA-event time of `run` on `stream`, a 256 MB buffer (> L2) rewritten before every
    launch so each one starts from a cold L2."""
    import torch

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=torch.cuda.current_device())
    times = []
    with torch.cuda.stream(stream):
        for i in range(warmup + steps):
            flush.zero_()
            # keep the stream busy while the host records the event and enqueues the launch, so
            # host-side launch latency never shows up between the two events
            torch.cuda._sleep(100_000)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run()
            e1.record(stream)
            if i >= warmup:
                times.append((e0, e1))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in times) / max(len(times), 1)


SWEEP_M = (1, 16, 128, 1024, 8192)
SWEEP_KN = ((2048, 8192), (8192, 2048), (2048, 2048), (768, 262144))


def gemm_sweep(args) -> int:
    """Benchmark config 3: the W8A8 GEMM (per-token activation scales, fp32 output) over
    M x (K, N), one JSON line per point against the roofline that bounds it: int8 tensor throughput
    (2 x measured bf16) or HBM bandwidth over the algorithmic bytes M*K + 4*M (activations) + N*K +
    4*N (weights) + 4*M*N (output). Two device timings per point, both CUDA events:
      - "isolated": one launch after a 256 MB L2 flush (cold L2, launch ramp and tail exposed);
      - "chain": back-to-back launches over R copies of the weight whose total exceeds twice the
        L2, captured as one CUDA graph, per-launch average (the decode pattern: one GEMM after
        another, every weight from HBM).
    Beside them the reference's quantise + GEMM region (e2ref_linear, E2_I8_BLOCK = K) on the host
    cores, best of 3, as GMAC/s and GB/s. E2C_SWEEP_M=1,16 restricts the token counts."""
    import ctypes as C

    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import oracle_ffi as of

    e2c = load_pkg()
    import e2c_b200.synthetic as syn

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    p = peaks()
    int8_peak, hbm = 2.0 * p["bf16_tflops"] * 1e12, p["hbm_gbs"] * 1e9
    lib = e2c.lib()
    lib.e2c_gemm_last_kernel.restype = C.c_char_p
    lib.e2c_gemm_ws_bytes.argtypes = [C.c_int]
    lib.e2c_gemm_ws_bytes.restype = C.c_size_t
    lib.e2cu_status.restype = C.c_void_p
    ms_only = [int(v) for v in os.environ.get("E2C_SWEEP_M", "").split(",") if v] or list(SWEEP_M)
    for K, N in SWEEP_KN:
        rng = np.random.default_rng(0xE2C0DE + 3 + K + N)
        wf = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        wq, wsc = syn.quantize_weight_rows(wf)
        ref = of.ref(K) if not args.no_cpu_baseline else None
        wref = of.Weight(wf, K, lib=ref) if ref is not None else None
        del wf
        copies = max(1, min(64, -(-(2 * 128 << 20) // (N * K))))
        Ws = [e2c.Weight(w=wq, scale=wsc) for _ in range(copies)]
        for M in ms_only:
            x = syn.activations(np.random.default_rng(M + K + N), M, K)
            qa, qs = e2c.quantize_rows(torch.from_numpy(x).to(dev), K)
            y = torch.empty((M, N), dtype=torch.float32, device=dev)
            wsb = lib.e2c_gemm_ws_bytes(M)
            wsp = torch.zeros(max(wsb // 4, 1) + 32, dtype=torch.int32, device=dev)
            argl = []
            for W in Ws:
                a = e2c.gemm_args(W, qa, qs, M)
                a.epi, a.y, a.ldy = e2c.EPI_F32, y.data_ptr(), N
                a.status = lib.e2cu_status()
                if wsb:
                    a.ws, a.ws_bytes = wsp.data_ptr(), wsb
                argl.append(a)
            ms, ms_chain, kernel = _gemm_point(e2c, lib, argl, stream, args.warmup, args.steps)
            ops = 2.0 * M * N * K
            nbytes = M * K + 4 * M + N * K + 4 * N + 4 * M * N
            t_tc, t_hbm = ops / int8_peak, nbytes / hbm

            def fr(ms_):
                t = ms_ / 1e3
                return {"us": round(ms_ * 1e3, 2), "tops": round(ops / t / 1e12, 1), "gbs": round(nbytes / t / 1e9, 1),
                        "frac_of_roofline": round(max(t_tc, t_hbm) / t, 3)}

            cpu = None
            if wref is not None:
                qa_c = np.empty((M, K), np.int8)
                as_c = np.empty((M, 1), np.float32)
                y_c = np.empty((M, N), np.float32)
                nthreads = ref.e2ref_init(0)
                t = _best_cpu(lambda: ref.e2ref_linear(x.ctypes.data_as(of.f32p), M, K, C.byref(wref.q),
                                                       qa_c.ctypes.data_as(of.i8p), as_c.ctypes.data_as(of.f32p),
                                                       y_c.ctypes.data_as(of.f32p)), warmup=1, reps=3, budget_s=15.0)
                cpu = {"us": round(t * 1e6, 1), "gmacs": round(M * N * K / t / 1e9, 1),
                       "gbs": round(nbytes / t / 1e9, 1), "threads": nthreads,
                       "what": "e2ref_linear: e2_quantize_blocks_avx512 + e2_i8_gemm_avx512 over the reference pool"}
            print(json.dumps({"sweep": "config 3", "M": M, "K": K, "N": N, "kernel": kernel,
                              "bound": "tensor" if t_tc > t_hbm else "hbm", "isolated": fr(ms), "chain": fr(ms_chain),
                              "chain_weights": len(argl), "pdl": os.environ.get("E2C_PDL") == "1" or kernel.endswith("_coresident"),
                              "peak_src": p["src"], "cpu_reference": cpu}), flush=True)
            del qa, qs, y, wsp, argl
        for W in Ws:
            W.free()
        del wref
    return 0


def _gemm_point(e2c, lib, argl, stream, warmup: int, steps: int):
    """(isolated ms, chain ms, kernel family) of one GEMM: the first launch alone after an L2 flush,
    and the per-launch average of back-to-back launches over every argument block in argl (one per
    weight copy) captured as one CUDA graph, so host launch overhead never paces the chain."""
    import torch

    ms = timed_launches(lambda: e2c.gemm_raw(argl[0], stream), stream, warmup, steps)
    kernel = lib.e2c_gemm_last_kernel().decode()
    e2c.check(stream)
    reps = max(2, min(64, (4 * steps) // len(argl)))
    with torch.cuda.stream(stream):
        for a in argl:
            e2c.gemm_raw(a, stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(reps):
            for a in argl:
                e2c.gemm_raw(a, stream)
    with torch.cuda.stream(stream):
        graph.replay()
        torch.cuda._sleep(100_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    e2c.check(stream)
    ms_chain = e0.elapsed_time(e1) / (reps * len(argl))
    del graph
    return ms, ms_chain, kernel


def small_m_table(dev, stream, warmup: int = 3, steps: int = 20) -> dict:
    """north_star's small-activation GEMMs in the default run: benchmark config 3's three short
    weights at M = 1 and 16 tokens, per-token scales, fp32 output; per point the kernel family, the
    isolated and chained launch times and the fraction of the HBM roofline (the weight, read once,
    is the bound)."""
    import ctypes as C

    import torch

    e2c = load_pkg()
    import e2c_b200.synthetic as syn

    lib = e2c.lib()
    lib.e2c_gemm_last_kernel.restype = C.c_char_p
    lib.e2c_gemm_ws_bytes.argtypes = [C.c_int]
    lib.e2c_gemm_ws_bytes.restype = C.c_size_t
    lib.e2cu_status.restype = C.c_void_p
    hbm = peaks()["hbm_gbs"] * 1e9
    out = {}
    for K, N in ((2048, 8192), (8192, 2048), (2048, 2048)):
        rng = np.random.default_rng(0xE2C0DE + 3 + K + N)
        wq, wsc = syn.quantize_weight_rows((rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)))
        copies = max(1, min(64, -(-(2 * 128 << 20) // (N * K))))
        Ws = [e2c.Weight(w=wq, scale=wsc) for _ in range(copies)]
        for M in (1, 16):
            x = syn.activations(np.random.default_rng(M + K + N), M, K)
            qa, qs = e2c.quantize_rows(torch.from_numpy(x).to(dev), K)
            y = torch.empty((M, N), dtype=torch.float32, device=dev)
            wsb = lib.e2c_gemm_ws_bytes(M)
            wsp = torch.zeros(max(wsb // 4, 1) + 32, dtype=torch.int32, device=dev)
            argl = []
            for W in Ws:
                a = e2c.gemm_args(W, qa, qs, M)
                a.epi, a.y, a.ldy = e2c.EPI_F32, y.data_ptr(), N
                a.status = lib.e2cu_status()
                if wsb:
                    a.ws, a.ws_bytes = wsp.data_ptr(), wsb
                argl.append(a)
            ms, ms_chain, kernel = _gemm_point(e2c, lib, argl, stream, warmup, steps)
            nbytes = M * K + 4 * M + N * K + 4 * N + 4 * M * N
            out[f"{K}x{N}_M{M}"] = {"kernel": kernel, "isolated_us": round(ms * 1e3, 2), "chain_us": round(ms_chain * 1e3, 2),
                                    "chain_frac_hbm": round(nbytes / hbm / (ms_chain / 1e3), 3),
                                    "isolated_frac_hbm": round(nbytes / hbm / (ms / 1e3), 3)}
            del qa, qs, y, wsp, argl
        for W in Ws:
            W.free()
    return out


if __name__ == "__main__":
    sys.exit(main())
