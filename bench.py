#!/usr/bin/env python
"""Benchmark of the B200 logits-to-token path on the batched-sampler workload.

Workload: B=32 rows x V=151,936 fp32 logits ~ N(0, 2.5^2) per GPU, per-row
parameters from a seed (T ~ U[0.3,1.2] with 25% greedy, top-k in {0,20,40,100}, top-p ~
U[0.7,1.0], repetition penalty ~ U[1.0,1.3], Adaptive mode), histories of 256-8,192 ids. A step is
one fused sampler launch (sixi_smp_sample) over one batch. Rows are independent, so N GPUs run
N batches with no collective (weak scaling); the timed region is bracketed by a barrier and
device synchronisation and its length is the max over ranks of the CUDA-event time.

  value         rows/s over all ranks, inputs resident in HBM (16 rotating batches, 311 MB per
                GPU > 126 MB L2, so every step reads its logits from HBM)
  e2e           rows/s through the host entry points: pinned host logits -> device -> tokens back,
                independent batches pipelined by sixi_smp_sample_host_async (the blocking
                sixi_smp_sample_host figure is reported beside it)
  roofline      algorithmic bytes per launch (logits + histories) / CUDA-event time per launch
  cpu_baseline  the engine's own CPU sampler (oracle/_ref) on all host threads, rank 0 at N=1

`--impl reference` times the engine's CPU sampler alone on the same workload (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "sixi-asi_b200"))

METRIC = "sampled rows/s at B=32,V=151,936 fp32; HBM GB/s vs B200 peak; 1/2/4/8 GPU"
UNIT = "rows/s"
ROWS = 32
VOCAB = 151_936
NBUF = 16
FALLBACK_HBM_GBS = 6650.0


def peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.tmp.flush()
        rows = []
        for line in Path(self.tmp.name).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append(f)
            except Exception:
                pass
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def make_batches(seed: int, rank: int = 0):
    """Config-2 batches: one parameter mix and history set (from `seed`, the same on every rank, so
    that every rank carries the same kind of work) and NBUF rotating logits batches per rank."""
    from sixi_smp import workloads as W

    base = W.config2(rows=ROWS, vocab=VOCAB, seed=seed)
    rng = np.random.default_rng(seed + 17 + 7919 * rank)
    first = base["logits"] if rank == 0 else W.config2_logits(rng, ROWS, VOCAB)
    logits = [first] + [W.config2_logits(rng, ROWS, VOCAB) for _ in range(NBUF - 1)]
    uniforms = [rng.random(ROWS) for _ in range(NBUF)]
    return base, logits, uniforms


def algorithmic_bytes(base: dict) -> int:
    return ROWS * VOCAB * 4 + 4 * int(base["hist_off"][-1])


def profiled_traffic(name: str = "row_kernel_sample_config2.md", key: str = "traffic_bytes_per_launch") -> int | None:
    """DRAM bytes (read + write) per row_kernel launch of a workload from its committed ncu summary
    (profiles/<name>, the line `<key>: <bytes>`), or None when it is absent."""
    import re

    p = REPO / "profiles" / name
    try:
        m = re.search(key + r":\s*(\d+)", p.read_text())
    except OSError:
        return None
    return int(m.group(1)) if m else None


def cpu_reference_rows_per_s(base, logits, uniforms, budget_s: float, n_threads: int = 0):
    """Times the engine's own CPU sampler (or the C restatement when the reference build is absent)
    on full batches until `budget_s` elapses. Returns (rows/s, kind, threads, sample text)."""
    from oracle import binding

    orc = binding.reference() or binding.port()
    threads = n_threads or os.cpu_count() or 1
    done = 0
    t0 = time.perf_counter()
    i = 0
    while True:
        orc.sample_batch(logits[i % len(logits)], base["params"], None, base["hist"], base["hist_off"],
                         uniforms[i % len(uniforms)], n_threads=threads)
        done += ROWS
        i += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return done / el, orc.kind, threads, f"{i} batches of {ROWS} rows ({el:.1f} s wall, {threads} threads)"


def run_reference(args) -> int:
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    base, logits, uniforms = make_batches(1000)
    from oracle import binding

    orc = binding.reference()
    kind = "reference"
    if orc is None:
        orc = binding.port()
        kind = "port"
    threads = os.cpu_count() or 1
    # size each step so that warmup + K steps stay within about 90 s
    t0 = time.perf_counter()
    orc.sample_batch(logits[0], base["params"], None, base["hist"], base["hist_off"], uniforms[0],
                     n_threads=threads)
    per_batch = time.perf_counter() - t0
    total_steps = max(1, args.steps + args.warmup)
    rows_per_step = ROWS
    if per_batch * total_steps > 90.0:
        rows_per_step = max(1, int(ROWS * 90.0 / (per_batch * total_steps)))
    lg = [np.ascontiguousarray(x[:rows_per_step]) for x in logits]
    prm = base["params"][:rows_per_step]
    hoff = base["hist_off"][:rows_per_step + 1]
    hist = base["hist"][:int(hoff[-1])]
    for i in range(args.warmup):
        orc.sample_batch(lg[i % NBUF], prm, None, hist, hoff, uniforms[i % NBUF][:rows_per_step], n_threads=threads)
    t0 = time.perf_counter()
    for i in range(args.steps):
        orc.sample_batch(lg[i % NBUF], prm, None, hist, hoff, uniforms[i % NBUF][:rows_per_step], n_threads=threads)
    el = time.perf_counter() - t0
    value = rows_per_step * args.steps / el
    sample = f"{rows_per_step} of {ROWS} rows per step, {args.steps} steps, {threads} threads"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "config2 batched sampler", "rows": ROWS, "vocab": VOCAB},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _graph_ms(step, steps: int, warmup: int, stream) -> float:
    """Runs `warmup` steps eagerly, captures `steps` steps in one CUDA graph and returns the CUDA-
    event time of its replay on `stream` (ms)."""
    import torch

    with torch.cuda.stream(stream):
        for i in range(warmup):
            step(i)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            step(i)
    with torch.cuda.stream(stream):
        graph.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1)


def run_workload(args) -> int:
    """The other configurations of the path on one GPU (reported beside the config-2 line):
    config1 single-row latency, config3 grammar-masked batch, config4 speculative verification,
    grammar: the JSON-constrained step with device-produced masks, numeric: the NaN / Inf policy
    pass over config-2 rows, drafter: batched suffix n-gram drafting."""
    import torch

    import sixi_smp as S
    from sixi_smp import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    peak, peak_kind = peaks()

    def t(x):
        if x is None:
            return None
        if x.dtype.names is not None:
            return torch.from_numpy(np.ascontiguousarray(x).view(np.uint8)).to(dev)
        if x.dtype == np.uint32:
            return torch.from_numpy(x.view(np.int32)).to(dev)
        if x.dtype == np.uint16:
            return torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
        return torch.from_numpy(np.ascontiguousarray(x)).to(dev)

    if args.workload in ("config1", "config3"):
        one = args.workload == "config1"
        rows = 1 if one else ROWS
        nbuf = NBUF
        if one:
            ds = [W.config1(seed=11 + i) for i in range(nbuf)]
            base = ds[0]
            logits = [t(x["logits"]) for x in ds]
        else:
            base = W.config3(rows=ROWS, vocab=VOCAB, seed=3)
            rng = np.random.default_rng(33)
            logits = [t(base["logits"])] + [t(W.config2_logits(rng, ROWS, VOCAB)) for _ in range(nbuf - 1)]
        params, masks = t(base["params"]), t(base["masks"])
        hist, hoff = t(base["hist"]), t(base["hist_off"])
        u = [torch.rand(rows, dtype=torch.float64, device=dev) for _ in range(nbuf)]
        smp = S.Sampler(0, 64, VOCAB)
        tok = torch.empty(rows, dtype=torch.int32, device=dev)
        sts = torch.empty(rows, dtype=torch.int32, device=dev)

        def step(i):
            smp.sample(logits[i % nbuf], params, masks=masks, hist=hist, hist_off=hoff, uniforms=u[i % nbuf],
                       out_tokens=tok, out_status=sts, stream=torch.cuda.current_stream())

        ms = _graph_ms(step, args.steps, args.warmup, stream)
        nbytes = rows * VOCAB * 4 + 4 * int(base["hist_off"][-1]) + (0 if masks is None else masks.numel() * 4)
        unit, value = ("us/step", 1e3 * ms / args.steps) if one else ("rows/s", rows * args.steps / (ms / 1e3))
        metric = ("single-row sampler step latency (config 1), V=151,936 fp32" if one else
                  "sampled rows/s at B=32,V=151,936 fp32 with grammar masks (config 3)")
        data = ("synthetic; 16 rotating rows (9.7 MB, L2-resident)" if one else
                "synthetic; 16 rotating batches (311 MB > L2), one mask set")
        launches = args.steps
    elif args.workload == "config4":
        streams, k = 32, 8
        nbuf = 2
        ds = [W.config4(streams=streams, k=k, vocab=VOCAB, seed=40 + i, stochastic=True, masked=True)
              for i in range(nbuf)]
        tgt = [t(x["target_bits"]) for x in ds]
        q = [t(x["q"]) for x in ds]
        dr = [t(x["drafts"]) for x in ds]
        params, masks = t(ds[0]["params"]), t(ds[0]["masks"])
        hist, hoff = t(ds[0]["hist"]), t(ds[0]["hist_off"])
        u = [t(x["uniforms"]) for x in ds]
        smp = S.Sampler(0, streams * (k + 1), VOCAB)

        def step(i):
            smp.verify(tgt[i % nbuf], dr[i % nbuf], params, draft_probs=q[i % nbuf], masks=masks, hist=hist,
                       hist_off=hoff, uniforms=u[i % nbuf], stream=torch.cuda.current_stream())

        ms = _graph_ms(step, args.steps, args.warmup, stream)
        # bytes the verifier must read: the target rows, q at each drafted id (the accept test), the
        # masks, drafts and histories. q is read further only where a draft is rejected (the
        # residual: at the kept candidates, or over the row on the top_k = 0 path), which this
        # count leaves out; the ncu capture (profiles/verify_config4_traffic.md) has the total.
        nbytes = (streams * (k + 1) * VOCAB * 2 + streams * k * 4 + masks.numel() * 4 + streams * k * 4 +
                  4 * int(ds[0]["hist_off"][-1]))
        unit, value = "stream-steps/s", streams * args.steps / (ms / 1e3)
        metric = "speculative verify stream-steps/s (config 4: S=32, k=8, V=151,936, bf16 target, fp32 q)"
        data = "synthetic; 2 rotating batches (491 MB > L2)"
        launches = 2 * args.steps  # row kernel + per-stream finalize
        extra = {}
        if not args.no_cpu:
            # the engine's own SpeculativeDecoder::step (slow path, dense q) per stream, on all host
            # threads, through the reference build's replay backend and fixed-draft drafter
            from oracle import binding as OB

            o = OB.reference()
            if o is not None and hasattr(o.lib, "orc_ref_spec_step_batch"):
                thr = os.cpu_count() or 1
                rs = np.stack([o.rng_seed(1000 + s) for s in range(streams)])
                n, i = 0, 0
                t0 = time.perf_counter()
                while time.perf_counter() - t0 < min(args.cpu_budget, 10.0):
                    x = ds[i % nbuf]
                    r = o.spec_step_batch(x["target_bits"], x["drafts"], ds[0]["params"], ds[0]["hist"],
                                          ds[0]["hist_off"], x["q"], rs, n_threads=thr)
                    assert (r["status"] == 0).all(), r["status"]
                    n += streams
                    i += 1
                el = time.perf_counter() - t0
                extra["cpu_baseline"] = {
                    "value": n / el, "unit": "stream-steps/s", "cores": thr, "kind": "reference",
                    "sample": (f"{i} batches of {streams} streams: the engine's SpeculativeDecoder::step (slow path, "
                               f"dense q, its own RNG) on the same target rows, drafts and q, {thr} threads; "
                               "the engine's step takes no grammar masks, so none are applied")}
    elif args.workload == "config4f":
        # the drafter -> verifier pipeline from draft logits: q = full_distribution(draft logits)
        # evaluated inside the verifier (sixi_smp_verify_draft_logits), beside the two-launch
        # pipeline that stores q first (sixi_smp_full_distribution + sixi_smp_verify)
        streams, k = 32, 8
        nbuf = 2
        ds = [W.config4(streams=streams, k=k, vocab=VOCAB, seed=40 + i, stochastic=True, masked=True)
              for i in range(nbuf)]
        tgt = [t(x["target_bits"]) for x in ds]
        dlg = [t(x["draft_logits"]) for x in ds]
        dr = [t(x["drafts"]) for x in ds]
        temps = torch.ones(streams * k, dtype=torch.float32, device=dev)
        params, masks = t(ds[0]["params"]), t(ds[0]["masks"])
        hist, hoff = t(ds[0]["hist"]), t(ds[0]["hist_off"])
        u = [t(x["uniforms"]) for x in ds]
        smp = S.Sampler(0, streams * (k + 1), VOCAB)
        qbuf = torch.empty((streams * k, VOCAB), dtype=torch.float32, device=dev)

        def step(i):
            smp.verify_draft_logits(tgt[i % nbuf], dlg[i % nbuf], temps, dr[i % nbuf], params, masks=masks,
                                    hist=hist, hist_off=hoff, uniforms=u[i % nbuf], stream=torch.cuda.current_stream())

        def step_stored(i):
            cs = torch.cuda.current_stream()
            q = smp.full_distribution(dlg[i % nbuf], temps, stream=cs)
            smp.verify(tgt[i % nbuf], dr[i % nbuf], params, draft_probs=q, masks=masks, hist=hist, hist_off=hoff,
                       uniforms=u[i % nbuf], stream=cs)

        ms = _graph_ms(step, args.steps, args.warmup, stream)
        ms_stored = _graph_ms(step_stored, args.steps, args.warmup, stream)
        # bytes that must be read: targets and draft logits in full (the statistics pass), masks,
        # drafts, histories
        nbytes = (streams * (k + 1) * VOCAB * 2 + streams * k * VOCAB * 4 + masks.numel() * 4 + streams * k * 4 +
                  4 * int(ds[0]["hist_off"][-1]))
        unit, value = "stream-steps/s", streams * args.steps / (ms / 1e3)
        metric = ("speculative verify from draft logits, stream-steps/s (S=32, k=8, V=151,936, bf16 target, "
                  "fp32 draft logits; q evaluated in the verifier)")
        data = "synthetic; 2 rotating batches (477 MB > L2)"
        launches = 3 * args.steps  # statistics pass + row kernel + per-stream finalize
        extra = {"stored_q_stream_steps_per_s": streams * args.steps / (ms_stored / 1e3),
                 "stored_q_ms_per_step": ms_stored / args.steps}
    elif args.workload == "grammar":
        from sixi_smp.json_grammar import JsonGrammar, Tokenizer, json_documents, json_vocab, prefix_states_tokens

        toks, flags, eos = json_vocab(VOCAB, seed=5)
        gram = JsonGrammar(0, toks, flags, eos)
        tk = Tokenizer(toks, flags)
        docs = json_documents(256, seed=21)
        nst = 4
        states = []
        for i in range(nst):  # rows spread over the automaton's modes, as decoding visits them
            pre, lens = prefix_states_tokens(docs, tk, ROWS, seed=100 + i)
            st = gram.new_states(ROWS)
            gram.advance(st, t(pre), t(lens))
            states.append(st)
        masks = torch.empty((ROWS, gram.mask_words), dtype=torch.int32, device=dev)

        def mask_step(i):
            gram.fill_masks(states[i % nst], out=masks, stream=torch.cuda.current_stream())

        mask_ms = _graph_ms(mask_step, args.steps, args.warmup, stream)
        # the whole constrained step: masks -> masked config-2 sampling -> automaton advance
        base = W.config2(rows=ROWS, vocab=VOCAB, seed=3)
        base["params"]["flags"] |= S.ROW_MASKED
        rng = np.random.default_rng(34)
        nbuf = NBUF
        logits = [t(base["logits"])] + [t(W.config2_logits(rng, ROWS, VOCAB)) for _ in range(nbuf - 1)]
        params, hist, hoff = t(base["params"]), t(base["hist"]), t(base["hist_off"])
        u = [torch.rand(ROWS, dtype=torch.float64, device=dev) for _ in range(nbuf)]
        smp = S.Sampler(0, 64, VOCAB)
        tok = torch.empty(ROWS, dtype=torch.int32, device=dev)
        sts = torch.empty(ROWS, dtype=torch.int32, device=dev)
        gst = torch.empty(ROWS, dtype=torch.int32, device=dev)
        live = gram.new_states(ROWS)

        def step(i):
            cs = torch.cuda.current_stream()
            if i % 64 == 0:  # start over from mid-document states now and then
                live.copy_(states[(i // 64) % nst])
            gram.fill_masks(live, out=masks, stream=cs)
            smp.sample(logits[i % nbuf], params, masks=masks, hist=hist, hist_off=hoff, uniforms=u[i % nbuf],
                       out_tokens=tok, out_status=sts, stream=cs)
            gram.advance(live, tok, out_status=gst, stream=cs)

        ms = _graph_ms(step, args.steps, args.warmup, stream)
        torch.cuda.synchronize()
        assert int((sts != 0).sum()) == 0 and int((gst != 0).sum()) == 0, (sts.tolist(), gst.tolist())
        vocab_bytes = 20 * VOCAB  # inline heads + meta words, L2-resident across rows and steps
        nbytes = (ROWS * VOCAB * 4 + 4 * int(base["hist_off"][-1]) + 2 * masks.numel() * 4 + vocab_bytes)
        unit, value = "rows/s", ROWS * args.steps / (ms / 1e3)
        metric = ("JSON-constrained sampled rows/s at B=32, V=151,936 fp32: device grammar masks + masked "
                  "sampling + automaton advance")
        data = ("synthetic; 16 rotating logits batches (311 MB > L2); synthetic 151,936-token vocabulary "
                "(L2-resident by design: read by every row of every step); states from prefixes of seeded "
                "JSON documents")
        launches = 3 * args.steps + args.steps // 64
        extra = {"mask_rows_per_s": ROWS * args.steps / (mask_ms / 1e3), "mask_us_per_batch": 1e3 * mask_ms / args.steps}
        if not args.no_cpu:
            from oracle import binding as OB

            o = OB.port()
            ov = OB.JsonVocab(toks, flags, eos)
            hs = states[0].cpu().numpy()
            thr = os.cpu_count() or 1
            t0 = time.perf_counter()
            n = 0
            while time.perf_counter() - t0 < min(args.cpu_budget, 10.0):
                OB.json_fill_masks(o, ov, hs, n_threads=thr)
                n += hs.shape[0]
            el = time.perf_counter() - t0
            extra["cpu_baseline"] = {"value": n / el, "unit": "mask rows/s", "cores": thr, "kind": "port",
                                     "sample": f"{n} rows of JSON-grammar masks (oracle automaton, {thr} threads)"}
        gram_obj = gram
    elif args.workload == "schema":
        from sixi_smp.json_grammar import json_vocab
        from sixi_smp.json_schema import SchemaGrammar

        toks, flags, eos = json_vocab(VOCAB, seed=5)
        gram = SchemaGrammar(0, W.RESPONSE_SCHEMA, toks, flags, eos)
        base = W.config2(rows=ROWS, vocab=VOCAB, seed=3)
        base["params"]["flags"] |= S.ROW_MASKED
        rng = np.random.default_rng(35)
        nbuf = NBUF
        logits = [t(base["logits"])] + [t(W.config2_logits(rng, ROWS, VOCAB)) for _ in range(nbuf - 1)]
        params, hist, hoff = t(base["params"]), t(base["hist"]), t(base["hist_off"])
        u = [torch.rand(ROWS, dtype=torch.float64, device=dev) for _ in range(nbuf)]
        smp = S.Sampler(0, 64, VOCAB)
        tok = torch.empty(ROWS, dtype=torch.int32, device=dev)
        sts = torch.empty(ROWS, dtype=torch.int32, device=dev)
        gst = torch.empty(ROWS, dtype=torch.int32, device=dev)
        masks = torch.empty((ROWS, gram.mask_words), dtype=torch.int32, device=dev)
        # row states as decoding visits them: constrained decoding from the start state, with
        # snapshots after 8, 24, 48 and 96 steps (rows whose answer ended start over)
        live = gram.new_states(ROWS)
        fresh = gram.new_states(ROWS)
        states = []
        with torch.cuda.stream(stream):
            for i in range(97):
                cs = torch.cuda.current_stream()
                gram.fill_masks(live, out=masks, stream=cs)
                smp.sample(logits[i % nbuf], params, masks=masks, hist=hist, hist_off=hoff, uniforms=u[i % nbuf],
                           out_tokens=tok, out_status=sts, step=i, stream=cs)
                gram.advance(live, tok, out_status=gst, stream=cs)
                done = (live[:, 0] == 0) & (live[:, 1] == 0) & (live[:, 2] == 0) & (live[:, 3] == 0)  # depth 0
                live.copy_(torch.where(done[:, None], fresh, live))
                if i in (8, 24, 48, 96):
                    states.append(live.clone())
        stream.synchronize()
        nst = len(states)

        def mask_step(i):
            gram.fill_masks(states[i % nst], out=masks, stream=torch.cuda.current_stream())

        mask_ms = _graph_ms(mask_step, args.steps, args.warmup, stream)

        def step(i):
            cs = torch.cuda.current_stream()
            if i % 64 == 0:  # start over from mid-answer states now and then
                live.copy_(states[(i // 64) % nst])
            gram.fill_masks(live, out=masks, stream=cs)
            smp.sample(logits[i % nbuf], params, masks=masks, hist=hist, hist_off=hoff, uniforms=u[i % nbuf],
                       out_tokens=tok, out_status=sts, step=i, stream=cs)
            gram.advance(live, tok, out_status=gst, stream=cs)

        ms = _graph_ms(step, args.steps, args.warmup, stream)
        torch.cuda.synchronize()
        ended = int((gst != 0).sum())  # rows whose answer ended inside a 64-step window (then masked out)
        vocab_bytes = 9 * VOCAB + int(sum(len(x) for x in toks))  # offsets, flags and token bytes: L2-resident
        nbytes = (ROWS * VOCAB * 4 + 4 * int(base["hist_off"][-1]) + 2 * masks.numel() * 4 + vocab_bytes)
        unit, value = "rows/s", ROWS * args.steps / (ms / 1e3)
        metric = ("json_schema-constrained sampled rows/s at B=32, V=151,936 fp32: device schema masks + masked "
                  "sampling + automaton advance")
        data = ("synthetic; 16 rotating logits batches (311 MB > L2); synthetic 151,936-token vocabulary; an "
                "order-extraction schema (nested objects, an unbounded array of objects, bounds, enums, a pattern, "
                "a format); row states from constrained decoding of random logits")
        launches = 3 * args.steps + args.steps // 64
        extra = {"mask_rows_per_s": ROWS * args.steps / (mask_ms / 1e3), "mask_us_per_batch": 1e3 * mask_ms / args.steps,
                 "rows_ended_in_window": ended,
                 "cpu_baseline": None,
                 "cpu_baseline_note": "none: the engine's json_schema automaton ships binary-only, so there is no "
                                      "reference CPU mask producer to time"}
        gram_obj = gram
    elif args.workload == "numeric":
        nbuf = NBUF
        rng = np.random.default_rng(51)
        logits = [t(W.config2_logits(rng, ROWS, VOCAB)) for _ in range(nbuf)]
        smp = S.Sampler(0, 64, VOCAB)
        rep = torch.empty((ROWS, 32), dtype=torch.uint8, device=dev)

        def step(i):
            smp.numeric_policy(logits[i % nbuf], S.NUMERIC_FAIL, 0.0, out=rep, stream=torch.cuda.current_stream())

        ms = _graph_ms(step, args.steps, args.warmup, stream)
        torch.cuda.synchronize()
        assert (S.numeric_reports(rep)["healthy"] == 1).all()
        nbytes = ROWS * VOCAB * 4 + ROWS * 32  # every logit read once, one report written per row
        unit, value = "rows/s", ROWS * args.steps / (ms / 1e3)
        metric = ("NaN/Inf policy rows/s at B=32, V=151,936 fp32 (inspect_and_apply_numeric_policy, "
                  "fail policy, read-only pass)")
        data = "synthetic; 16 rotating batches (311 MB > L2)"
        launches = args.steps
        extra = {}
        if not args.no_cpu:
            from oracle import binding as OB

            o = OB.reference() or OB.port()
            host = [x.cpu().numpy() for x in logits[:2]]
            n = 0
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < min(args.cpu_budget, 5.0):
                row = host[n % 2][n % ROWS].copy()
                o.numeric_policy(row, 0, 0.0)
                n += 1
            el = time.perf_counter() - t0
            extra["cpu_baseline"] = {"value": n / el, "unit": "rows/s", "cores": 1, "kind": o.kind,
                                     "sample": f"{n} rows of {VOCAB} fp32 (the engine's function, 1 thread)"}
    elif args.workload == "drafter":
        # 32 streams of 16,384-token histories: every fourth repeats a phrase (a match is found
        # early), the rest are random over the vocabulary (the engine then runs its exact-tail search
        # over the whole window)
        streams, hlen, k = ROWS, 16384, 8
        rng = np.random.default_rng(61)
        hs = []
        for i in range(streams):
            h = rng.integers(0, VOCAB, size=hlen).astype(np.int32)
            if i % 4 == 0:
                h[6000:6012] = h[-12:]
            hs.append(h)
        off = np.zeros(streams + 1, np.int64)
        off[1:] = np.cumsum([h.size for h in hs])
        d_hist, d_off = t(np.concatenate(hs)), t(off)
        smp = S.Sampler(0, 64, VOCAB)
        drafts = torch.empty((streams, k), dtype=torch.int32, device=dev)
        mlen = torch.empty(streams, dtype=torch.int32, device=dev)

        def step(i):
            smp.suffix_draft(d_hist, d_off, k=k, min_match_len=3, max_window_tokens=16384, out=drafts, out_match=mlen,
                             stream=torch.cuda.current_stream())

        ms = _graph_ms(step, args.steps, args.warmup, stream)
        torch.cuda.synchronize()
        assert (mlen.cpu().numpy()[::4] > 0).all()
        nbytes = 4 * int(off[-1])  # every history token read once
        unit, value = "stream-steps/s", streams * args.steps / (ms / 1e3)
        metric = ("suffix n-gram drafts per second: SuffixDrafter(3, 16384).propose for 32 streams of 16,384-token "
                  "histories, k = 8")
        data = "synthetic; random token histories, a quarter with a repeated 12-token phrase"
        launches = args.steps
        extra = {}
        if not args.no_cpu:
            from oracle import binding as OB

            o = OB.reference() or OB.port()
            n = 0
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < min(args.cpu_budget, 5.0):
                o.suffix_draft(hs[n % streams], 3, 16384, k)
                n += 1
            el = time.perf_counter() - t0
            extra["cpu_baseline"] = {"value": n / el, "unit": "stream-steps/s", "cores": 1, "kind": o.kind,
                                     "sample": f"{n} proposals of the engine's SuffixDrafter on these histories, 1 thread"}
    else:
        raise SystemExit(f"unknown workload {args.workload}")
    per_launch_s = ms / 1e3 / args.steps
    achieved = nbytes / per_launch_s / 1e9
    line = {
        "metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": unit != "us/step", "scaling": "weak", "vs_baseline": None,
        "dtype": ("bf16" if args.workload.startswith("config4") else ("int32" if args.workload == "drafter" else "f32")),
        "data": data,
        "config": {"workload": args.workload},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": ({"config4": profiled_traffic("verify_config4_traffic.md"),
                                  "numeric": profiled_traffic("numeric_kernel_config2.md")}.get(args.workload)),
                     "peak_source": peak_kind, "bytes_per_launch": int(nbytes)},
        "gpu_launches": launches,
    }
    if args.workload in ("grammar", "schema", "config4", "config4f", "numeric", "drafter"):
        line.update(extra)
    if args.workload in ("grammar", "schema"):
        gram_obj.close()
    print(json.dumps(line), flush=True)
    smp.close()
    return 0


def _init_dist(local: int, world: int):
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    return dev


def _max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_config5(args) -> int:
    """BASELINE config 5, rows partitioned: 8,192 rows x V = 151,936 fp32 (4.98 GB) with the
    config-2 parameter mix, split into N equal row ranges, one per rank (strong scaling: the total
    is fixed). A step is one sixi_smp_sample launch per rank over its rows; there is no collective
    in the timed region. The logits are drawn on the device (one buffer per rank, 622 MB at N = 8,
    larger than L2, so every step reads them from HBM)."""
    import torch
    import torch.distributed as dist

    import sixi_smp as S
    from sixi_smp import workloads as W

    rank, world, local = dist_env()
    dev = _init_dist(local, world)
    total = args.rows
    if total % world:
        raise SystemExit(f"--rows {total} is not a multiple of the {world} ranks")
    R = total // world
    mix = W.config2_mix(total, VOCAB, seed=5)
    prm = np.ascontiguousarray(mix["params"][rank * R:(rank + 1) * R])
    off = mix["hist_off"][rank * R:(rank + 1) * R + 1]
    hist = np.ascontiguousarray(mix["hist"][off[0]:off[-1]])
    off = off - off[0]
    logits = W.config2_logits_device(R, VOCAB, seed=5000 + rank, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    u = torch.rand(R, dtype=torch.float64, device=dev, generator=g)
    d_params = torch.from_numpy(prm.view(np.uint8)).to(dev)
    d_hist, d_hoff = torch.from_numpy(hist).to(dev), torch.from_numpy(off).to(dev)
    smp = S.Sampler(local, R, VOCAB)
    tok = torch.empty(R, dtype=torch.int32, device=dev)
    sts = torch.empty(R, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(i):
        smp.sample(logits, d_params, hist=d_hist, hist_off=d_hoff, uniforms=u, step=i, out_tokens=tok,
                   out_status=sts, stream=torch.cuda.current_stream())

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    stream.synchronize()
    assert int((sts != 0).sum()) == 0, "non-zero statuses"
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(args.steps):
            step(i)
    with torch.cuda.stream(stream):
        graph.replay()
    stream.synchronize()
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.05)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_max = _max_over_ranks(ms, world, dev)
    value = total * args.steps / (ms_max / 1e3)
    nbytes = R * VOCAB * 4 + 4 * int(off[-1])
    achieved = nbytes / (ms / args.steps / 1e3) / 1e9
    peak, peak_kind = peaks()

    # end to end through the host entry point: this rank's rows from pinned host memory
    e2e = None
    n_e2e = min(args.e2e_steps, 3)
    if n_e2e > 0:
        h_logits = torch.empty((R, VOCAB), dtype=torch.float32).pin_memory()
        h_logits.copy_(logits)
        h_np = h_logits.numpy()
        pin = lambda a: torch.from_numpy(a).pin_memory().numpy()  # noqa: E731
        h_params = pin(prm.view(np.uint8)).view(S.PARAMS_DTYPE)
        h_hist, h_hoff, h_u = pin(hist), pin(off), pin(u.cpu().numpy())
        h_tok = pin(np.empty(R, np.int32))
        h_st = pin(np.empty(R, np.int32))
        smp.sample_host(h_np, h_params, hist=h_hist, hist_off=h_hoff, uniforms=h_u, out_tokens=h_tok,
                        out_status=h_st, stream=stream)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            smp.sample_host(h_np, h_params, hist=h_hist, hist_off=h_hoff, uniforms=h_u, out_tokens=h_tok,
                            out_status=h_st, stream=stream)
        el = _max_over_ranks(time.perf_counter() - t0, world, dev)
        e2e = {"value": total * n_e2e / el, "unit": "rows/s",
               "h2d_bytes_per_step": int(h_np.nbytes + h_params.nbytes + h_hist.nbytes + h_hoff.nbytes + h_u.nbytes),
               "d2h_bytes_per_step": int(h_tok.nbytes + h_st.nbytes)}
        del h_logits

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        base, lg, us = make_batches(1000)
        v, kind, threads, sample = cpu_reference_rows_per_s(base, lg, us, args.cpu_budget)
        cpu = {"value": v, "unit": "rows/s", "cores": threads, "kind": kind,
               "sample": sample + "; config-2 batches (the same parameter mix)"}
    if world > 1:
        del graph
        dist.barrier()
        dist.destroy_process_group()
    t1024 = profiled_traffic("config5_sharded_splits.md", key="traffic_bytes_per_1024_rows")
    traffic = int(t1024 * R / 1024) if t1024 else None
    if rank == 0:
        line = {
            "metric": "sampled rows/s, 8,192 rows x V=151,936 fp32 partitioned over N GPUs (config 5)",
            "value": value, "unit": "rows/s", "tokens_per_s": value, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic; logits drawn on the device (N(0, 2.5^2), 16 ids per row +8), config-2 mix",
            "config": {"workload": "config5 rows partitioned", "rows_total": total, "rows_per_gpu": R,
                       "vocab": VOCAB, "parallelism": f"rows partitioned, {world} GPU(s), no collective",
                       "l2": f"inputs larger than L2: {R * VOCAB * 4 / 1e6:.0f} MB of logits per GPU"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "bytes_per_launch": int(nbytes),
                         "traffic_note": "ncu DRAM bytes of a 1,024-row launch of the same mix, scaled to this "
                                         "rank's rows (profiles/config5_sharded_splits.md)"},
            "e2e": e2e, "cpu_baseline": cpu, "gpu_launches": args.steps, "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    smp.close()
    return 0


def run_config5_sharded(args) -> int:
    """BASELINE config 5, vocab-sharded variant: B = 256 rows whose vocabulary is split into equal
    slices (8 on one GPU, emulated as 8 slices of the rows; one per rank on N > 1 GPUs). A step is
    stage 1 on each slice (per-slice top-64 candidates and softmax statistics), the exchange
    (NCCL all-gather over NVLink on N > 1; a stack of the slices' outputs on one GPU), stage 2 (the
    merge, identical on every rank) and round 2 for the rows the merge cannot certify. CUDA events
    split each step into those four parts; the reported time is their sum, max over ranks."""
    import torch
    import torch.distributed as dist

    import sixi_smp as S
    from sixi_smp import workloads as W
    from sixi_smp.sharded import ShardLayout, sample_vocab_sharded

    rank, world, local = dist_env()
    dev = _init_dist(local, world)
    B, top_n = 256, 64
    n_shards = 8 if world == 1 else world
    lay = ShardLayout(VOCAB, n_shards)
    mix = W.config2_mix(B, VOCAB, seed=6)
    full = W.config2_logits_device(B, VOCAB, seed=6000, device=dev)
    params = torch.from_numpy(mix["params"].view(np.uint8)).to(dev)
    hist, hoff = torch.from_numpy(mix["hist"]).to(dev), torch.from_numpy(mix["hist_off"]).to(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    u = torch.rand(B, dtype=torch.float64, device=dev, generator=g)
    smp = S.Sampler(local, 4096, VOCAB)
    stream = torch.cuda.Stream(device=dev)
    parts = ("stage1", "exchange", "stage2", "round2")
    if world > 1:
        mine = full[:, lay.offset(rank):lay.offset(rank) + lay.width(rank)].contiguous()
        del full
    else:
        slices = [full[:, lay.offset(r):lay.offset(r) + lay.width(r)].contiguous() for r in range(n_shards)]

    def one_step(i, ev):
        def mark(name):
            ev[name].record(torch.cuda.current_stream())

        if world > 1:
            return sample_vocab_sharded(mine, lay, rank, params, top_n=top_n, hist=hist, hist_off=hoff, uniforms=u,
                                        step=i, sampler=smp, stream=torch.cuda.current_stream(), mark=mark)
        cs = torch.cuda.current_stream()
        cands, stats = [], []
        for r in range(n_shards):
            c, s = smp.shard_candidates(slices[r], lay.offset(r), lay.width(r), params, top_n=top_n, hist=hist,
                                        hist_off=hoff, stream=cs)
            cands.append(c)
            stats.append(s)
        mark("stage1")
        gc, gs = torch.stack(cands), torch.stack(stats)
        mark("exchange")
        tok, sts = smp.merge_shards(gc, gs, params, uniforms=u, step=i, stream=cs)
        mark("stage2")
        rows = (sts == 2).nonzero().flatten().to(torch.int32)
        if rows.numel():
            fr = torch.empty((rows.numel(), VOCAB), dtype=torch.float32, device=dev)
            for r in range(n_shards):  # each slice's flagged rows into its columns of the rebuilt rows
                smp.gather_rows(slices[r], rows, lay.width(r), out=fr[:, lay.offset(r):], stream=cs)
            smp.sample_indexed(fr, rows, params, tok, sts, hist=hist, hist_off=hoff, uniforms=u, step=i, stream=cs)
        mark("round2")
        return tok, sts

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            ev = {k: torch.cuda.Event(enable_timing=True) for k in ("start",) + parts}
            ev["start"].record(stream)
            tok, sts = one_step(i, ev)
    stream.synchronize()
    n_round2 = int((sts == 2).sum())  # should be 0 after round 2
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.05)
    evs = []
    flagged = []
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            ev = {k: torch.cuda.Event(enable_timing=True) for k in ("start",) + parts}
            ev["start"].record(stream)
            tok, sts = one_step(i, ev)
            evs.append(ev)
    torch.cuda.synchronize()
    clk = clocks.stop()
    split = {k: 0.0 for k in parts}
    for ev in evs:
        prev = ev["start"]
        for k in parts:
            split[k] += prev.elapsed_time(ev[k])
            prev = ev[k]
    split = {k: v / args.steps for k, v in split.items()}
    ms_step = sum(split.values())
    ms_max = _max_over_ranks(ms_step, world, dev)
    # rows the merge sent to round 2 in the last step (recounted without round 2)
    with torch.cuda.stream(stream):
        ev = {k: torch.cuda.Event(enable_timing=True) for k in ("start",) + parts}
        if world > 1:
            c, s = smp.shard_candidates(mine, lay.offset(rank), lay.width(rank), params, top_n=top_n, hist=hist,
                                        hist_off=hoff, stream=stream)
            gc = torch.empty((world,) + tuple(c.shape), dtype=c.dtype, device=dev)
            gs = torch.empty((world,) + tuple(s.shape), dtype=s.dtype, device=dev)
            dist.all_gather_into_tensor(gc.view(-1, *c.shape[1:]), c)
            dist.all_gather_into_tensor(gs.view(-1, *s.shape[1:]), s)
        else:
            cs_ = [smp.shard_candidates(slices[r], lay.offset(r), lay.width(r), params, top_n=top_n, hist=hist,
                                        hist_off=hoff, stream=stream) for r in range(n_shards)]
            gc, gs = torch.stack([c for c, _ in cs_]), torch.stack([s for _, s in cs_])
        _, s1 = smp.merge_shards(gc, gs, params, uniforms=u, stream=stream)
    stream.synchronize()
    flagged = int((s1 == 2).sum())
    payload = int(gc[0].numel() * gc.element_size() + gs[0].numel() * gs.element_size())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        w = lay.width(0)
        nbytes = B * w * 4 + 4 * int(mix["hist_off"][-1])
        line = {
            "metric": "vocab-sharded sampled rows/s, B=256, V=151,936 fp32 split into equal slices (config 5)",
            "value": B / (ms_max / 1e3), "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic; config-2 mix, logits drawn on the device",
            "config": {"workload": "config5 vocab-sharded", "rows": B, "vocab": VOCAB, "slices": n_shards,
                       "top_n": top_n, "parallelism": (f"vocab-sharded over {world} GPUs, NCCL all-gather" if world > 1
                                                       else "8 slices emulated on 1 GPU, no collective")},
            "split_ms_per_step": split, "rows_to_round2_per_step": flagged,
            "exchange_payload_bytes_per_rank": payload, "unresolved_after_round2": n_round2,
            "roofline": {"bound": "hbm", "achieved": nbytes / (ms_step / 1e3) / 1e9 if world > 1 else
                         n_shards * nbytes / (ms_step / 1e3) / 1e9, "unit": "GB/s",
                         "note": "stage-1 bytes of this rank's slice (all slices on 1 GPU) over the whole step"},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    smp.close()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--workload", default="config2", choices=["config2", "config1", "config3", "config4", "config4f",
                                                                 "config5", "config5s", "grammar", "schema", "numeric",
                                                                 "drafter"],
                    help="config2 is the headline line; the others are reported beside it (config5 and config5s "
                         "also under torchrun on N GPUs)")
    ap.add_argument("--rows", type=int, default=8192, help="config5: total rows over all ranks")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "config5":
        return run_config5(args)
    if args.workload == "config5s":
        return run_config5_sharded(args)
    if args.workload != "config2":
        return run_workload(args)

    import torch
    import torch.distributed as dist

    import sixi_smp as S

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    base, logits, uniforms = make_batches(1000, rank)
    d_logits = [torch.from_numpy(x).to(dev) for x in logits]
    d_u = [torch.from_numpy(u).to(dev) for u in uniforms]
    d_params = torch.from_numpy(base["params"].view(np.uint8)).to(dev)
    d_hist = torch.from_numpy(base["hist"]).to(dev)
    d_hoff = torch.from_numpy(base["hist_off"]).to(dev)
    smp = S.Sampler(local, 1024, VOCAB)
    tok = torch.empty(ROWS, dtype=torch.int32, device=dev)
    sts = torch.empty(ROWS, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(i: int, s) -> None:
        smp.sample(d_logits[i % NBUF], d_params, hist=d_hist, hist_off=d_hoff, uniforms=d_u[i % NBUF],
                   out_tokens=tok, out_status=sts, stream=s)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i, stream)
    stream.synchronize()
    assert int((sts != 0).sum()) == 0, f"statuses {sts.tolist()}"
    # the K timed steps are captured once in a CUDA graph (launch-bound otherwise: one ~6 us launch
    # per step from Python)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(args.steps):
            step(i, torch.cuda.current_stream())
    # CUDAGraph.replay() launches on the current stream: replay and time inside `stream`
    with torch.cuda.stream(stream):
        graph.replay()
    stream.synchronize()

    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.05)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    value = world * ROWS * args.steps / (ms_max / 1e3)

    # roofline of the fused launch (this rank)
    bytes_per_launch = algorithmic_bytes(base)
    achieved = bytes_per_launch / (ms / args.steps / 1e3) / 1e9
    peak, peak_kind = peaks()

    # end to end through the host entry points: pinned host logits in, tokens out. `e2e` pipelines
    # independent batches through sixi_smp_sample_host_async (two staging slots: batch i+1's
    # host->device copy overlaps batch i's kernel; every batch's tokens are copied back); the
    # blocking sixi_smp_sample_host (one synchronised call per batch) is reported beside it.
    e2e = None
    if args.e2e_steps > 0:
        pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()  # noqa: E731
        h_lg = [pin(logits[0]), pin(logits[1])]
        h_params = pin(base["params"].view(np.uint8)).view(S.PARAMS_DTYPE)
        h_hist, h_hoff = pin(base["hist"]), pin(base["hist_off"])
        h_u = [pin(uniforms[0]), pin(uniforms[1])]
        h_tok = [pin(np.empty(ROWS, np.int32)) for _ in range(2)]
        h_st = [pin(np.empty(ROWS, np.int32)) for _ in range(2)]

        def host_step(i, wait):
            smp.sample_host(h_lg[i % 2], h_params, hist=h_hist, hist_off=h_hoff, uniforms=h_u[i % 2],
                            out_tokens=h_tok[i % 2], out_status=h_st[i % 2], stream=stream, wait=wait)

        def timed(wait):
            for i in range(3):
                host_step(i, wait)
            stream.synchronize()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for i in range(args.e2e_steps):
                host_step(i, wait)
            stream.synchronize()
            el = time.perf_counter() - t0
            assert int(h_st[0].sum()) == 0 and int(h_st[1].sum()) == 0
            if world > 1:
                t = torch.tensor([el], device=dev, dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                el = float(t.item())
            return world * ROWS * args.e2e_steps / el

        v_pipe = timed(False)
        v_block = timed(True)
        h2d = h_lg[0].nbytes + h_params.nbytes + h_hist.nbytes + h_hoff.nbytes + h_u[0].nbytes
        e2e = {"value": v_pipe, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(h_tok[0].nbytes + h_st[0].nbytes),
               "mode": "sixi_smp_sample_host_async over independent batches (2 staging slots)",
               "blocking_value": v_block}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, kind, threads, sample = cpu_reference_rows_per_s(base, logits, uniforms, args.cpu_budget)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample}

    if world > 1:
        del graph
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config2 batched sampler", "rows_per_gpu": ROWS, "vocab": VOCAB,
                       "parallelism": f"rows partitioned, {world} GPU(s), no collective",
                       "l2": f"inputs larger than L2: {NBUF} rotating batches, "
                             f"{NBUF * ROWS * VOCAB * 4 / 1e6:.0f} MB per GPU"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profiled_traffic(), "peak_source": peak_kind,
                         "bytes_per_launch": bytes_per_launch},
            "e2e": e2e,
            "cpu_baseline": cpu,
            "gpu_launches": args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    smp.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
