"""Benchmark: full constrained beam search throughput (seq*beams/s) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg5] [--impl b200|reference]

A step = one full L-level constrained beam search over this rank's shard of
the workload (config 5 by default: 16M-item catalog, H=3584, bf16, batch
65,536 x 10 beams, top-k 10; `--workload cfg4` is the Gumbel-max sampled
search), plus -- for N > 1 -- the NCCL all-gather of every rank's results.
Inputs (trie, head rows, per-level hidden states) are resident in HBM before
timing.  One search is captured as a CUDA graph and replayed K times after W
warm-ups, timed with CUDA events on the launching stream.  At config 5 the
hidden states (10 GB at N=1) exceed the 126 MB L2; smaller workloads get a
256 MB write before every timed replay (timed separately and subtracted).
value = (sum over levels of rows) * N / (max over ranks of the device time
per step).

`e2e` runs the same search through the public API with the hidden states in
pinned host memory, host->device copies (overlapped with compute) and the
device->host copy of the results inside the timed region.

`--impl reference` times the CPU restatement of the reference's algorithm
(oracle/vtnk_oracle.py, the reference itself is Python and is not installed
on the GPU box) on a bounded sample of the same workload with all host threads.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "constrained beam-step seq*beams/s (full L-level search)"
UNIT = "seq*beams/s"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        if not self.lines:  # very short timed region: take one reading now
            try:
                r = subprocess.run(["nvidia-smi", f"--query-gpu={self.FIELDS}",
                                    "--format=csv,noheader,nounits", "-i", str(self.gpu)],
                                   capture_output=True, text=True, timeout=10)
                self.lines += r.stdout.strip().splitlines()
            except (OSError, subprocess.TimeoutExpired):
                pass
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- algorithmic cost
def level_costs(w, dw, curs, wins):
    """Algorithmic bytes and flops of each level's step kernel (per launch)."""
    import torch

    rp = dw.trie.row_ptrs
    nnz = dw.trie.stacked_cols_vals.shape[1] - 1
    es = 4 if w.dtype == "f32" else 2
    out = []
    for level, cur in enumerate(curs):
        rows = dw.hidden[level].shape[0]
        if cur is None:
            uniq = torch.zeros(1, dtype=torch.long, device=rp.device)
        else:
            uniq = torch.unique(cur)
        nxt = torch.where(uniq + 1 < rp.numel(), rp[(uniq + 1).clamp(max=rp.numel() - 1)],
                          torch.full_like(uniq, nnz))
        kids_unique = int((nxt - rp[uniq]).clamp(min=0).sum())
        if cur is None:
            kids_rows = kids_unique * rows
        else:
            c = cur
            cn = torch.where(c + 1 < rp.numel(), rp[(c + 1).clamp(max=rp.numel() - 1)],
                             torch.full_like(c, nnz))
            kids_rows = int((cn - rp[c]).clamp(min=0).sum())
        bytes_ = (rows * w.hidden * es                       # hidden states
                  + uniq.numel() * 16 + kids_unique * 16     # CSR rows touched (row_ptr pair, col+val)
                  + wins[level][1] * w.hidden * es           # level head slice
                  + (rows * (4 + 8) if w.sampling                  # sample + node
                     else rows * w.topk * (4 + 8 + 8) + rows * 4))  # candidates + row lse
        flops = 2 * w.hidden * kids_rows
        out.append((bytes_, flops))
    return out


# --------------------------------------------------------------------------- CPU baseline
class CpuBaseline:
    """The oracle's beam search (fp32, the reference's sparse path) on a
    bounded sample of queries of workload ``w``, parallel over query chunks."""

    def __init__(self, w):
        from oracle import vtnk_oracle as O
        from rectokens_b200 import synthetic as S

        self.w, self.O, self.S = w, O, S
        tok = S.to_tokens(w.make_catalog(), w.codes)
        self.rp, self.cv, self.lmb, _, _ = O.build_sorted_csr(tok, w.vocab, 1)
        self.W = (S.head_f32(w.seed, w.vocab, w.hidden) if w.dtype == "f32"
                  else S.bf16_bits_to_f32(S.head_bits(w.seed, w.vocab, w.hidden)))

    def _hidden(self, level, q0, nq):
        w, S = self.w, self.S
        r0, rows = (q0, nq) if level == 0 else (q0 * w.beams, nq * w.beams)
        if w.dtype == "f32":
            return S.hidden_f32(w.seed, level, r0, rows, w.hidden)
        return S.bf16_bits_to_f32(S.hidden_bits(w.seed, level, r0, rows, w.hidden))

    def _sample_search(self, hidden, q0):
        """The reference's sampling op level by level (kernels:562-783): Gumbel
        noise at the rows' global offsets, argmax, next node of the sample."""
        O, w = self.O, self.w
        cur = np.zeros(hidden[0].shape[0], dtype=np.int64)
        for level, a in enumerate(hidden):
            mb = self.lmb[level]
            noise = O.gumbel_noise(w.seed, a.shape[0], mb, row0=q0)
            nn, _, smp, score = O.fused_sampling(a, self.W.T, None, self.rp, self.cv, cur, mb,
                                                 noise, w.temperature, acc=np.float32)
            best = np.argmax(score, axis=1)
            cur = np.where(smp >= 0, nn[np.arange(nn.shape[0]), best], -1)
        return cur

    def rows(self, nq):
        return nq * (1 + self.w.beams * (self.w.levels - 1))

    def run(self, nq, threads, q0=0):
        """Seconds for queries [q0, q0 + nq) (input generation not timed)."""
        w = self.w
        per = max(1, -(-nq // threads))
        chunks = [(q, min(per, q0 + nq - q)) for q in range(q0, q0 + nq, per)]
        inputs = {c: [self._hidden(l, *c) for l in range(w.levels)] for c in chunks}

        def one(c):
            if w.sampling:
                self._sample_search(inputs[c], c[0])
            else:
                self.O.beam_search(inputs[c], self.W, self.rp, self.cv, self.lmb, c[1], w.beams,
                                   w.topk, acc=np.float32)

        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(one, chunks))
        return time.perf_counter() - t0


# --------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="cfg5")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the workload's query count (smaller cases for profiling)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-queries", type=int, default=0,
                    help="queries in the CPU-baseline sample (0 = auto)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    from rectokens_b200 import synthetic as S

    w = S.WORKLOADS[args.workload]
    if args.batch:
        import dataclasses

        w = dataclasses.replace(w, batch=args.batch)
    workload_cfg = {
        "workload": (f"{args.workload}: {w.levels}-level Gumbel-max sampled search "
                     f"(T={w.temperature}, Philox seed {w.seed}), catalog K={w.codes} "
                     f"L={w.levels}, H={w.hidden} {w.dtype} head, batch {w.batch}"
                     if w.sampling else
                     f"{args.workload}: {w.levels}-level beam search, catalog K={w.codes} "
                     f"L={w.levels}, H={w.hidden} {w.dtype} head, batch {w.batch} x {w.beams} "
                     f"beams, top-{w.topk}"),
        "global_batch": w.batch, "beams": w.beams, "topk": w.topk, "levels": w.levels,
        "hidden": w.hidden, "rows_per_search": S.search_rows(w),
        "parallelism": f"dp{args.gpus}" if args.gpus > 1 else "single",
    }

    if args.impl == "reference":
        if rank != 0:
            return
        threads = os.cpu_count() or 1
        cpu = CpuBaseline(w)
        probe = threads * 2
        rate0 = cpu.rows(probe) / cpu.run(probe, threads)
        per_step_s = min(30.0, max(2.0, 150.0 / max(1, args.steps + args.warmup)))
        nq = args.cpu_queries or max(threads, int(per_step_s * rate0 / cpu.rows(1)))
        nq = min(nq, w.batch)
        for i in range(args.warmup):
            cpu.run(nq, threads, q0=i * nq)
        times = [cpu.run(nq, threads, q0=(args.warmup + i) * nq) for i in range(args.steps)]
        rate = cpu.rows(nq) * len(times) / sum(times)
        sample = (f"{nq} queries per step of {args.workload} (all {w.levels} levels, "
                  f"{cpu.rows(nq)} rows, {statistics.mean(times):.1f} s per step)")
        line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT,
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1e3 * statistics.mean(times),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 (bf16 inputs upcast, as the reference's CPU path)",
                "data": "synthetic (seeded catalog / head / hidden states)", "config": workload_cfg,
                "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                                 "sample": sample},
                "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    from rectokens_b200 import workload as WL
    from rectokens_b200.distributed import ResultRecord
    from rectokens_b200.decoding.beam_search import (
        beam_merge,
        beam_step,
        _search_struct,
        constrained_beam_search_from_host,
        constrained_sampling_search,
        child_index,
        level_windows,
    )
    from rectokens_b200.schemas import GenerationConfig
    from rectokens_b200 import _lib as L

    cfg = GenerationConfig(steps=w.levels, k=w.beams, beam_size=w.topk, temperature=0.0)
    dw = WL.make_device_workload(w, dev, shard=rank, n_shards=world)
    wins = level_windows(dw.trie)
    idxs = [child_index(dw.trie, l) for l in range(w.levels)]
    Bq, k = dw.batch, w.beams

    # preallocated per-level buffers: the timed loop allocates nothing
    rows_l = [h.shape[0] for h in dw.hidden]
    lib = L.lib()
    csr = L.csr_struct(dw.trie.row_ptrs, dw.trie.stacked_cols_vals)
    bufs = []
    for level, R in enumerate(rows_l):
        bufs.append(dict(
            tok=torch.empty((R, w.topk), dtype=torch.int64, device=dev),
            logit=torch.empty((R, w.topk), dtype=torch.float32, device=dev),
            node=torch.empty((R, w.topk), dtype=torch.int64, device=dev),
            lse=torch.empty((R,), dtype=torch.float32, device=dev),
            ids=torch.empty((Bq * k, level + 1), dtype=torch.int64, device=dev),
            logp=torch.empty((Bq * k,), dtype=torch.float32, device=dev),
            nxt=torch.empty((Bq * k,), dtype=torch.int64, device=dev),
            parent=torch.empty((Bq * k,), dtype=torch.int64, device=dev)))
    lins = [L.linear_struct(dw.hidden[l], dw.weight.T, None) for l in range(w.levels)]
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    # the last level writes its results straight into this rank's packed
    # record, which one all-gather concatenates across ranks
    rec = ResultRecord(Bq * k, w.levels, dev)
    bufs[-1]["ids"], bufs[-1]["logp"], bufs[-1]["nxt"] = rec.ids, rec.logp, rec.node
    gather_buf = (torch.empty((world * rec.nbytes,), dtype=torch.uint8, device=dev)
                  if world > 1 else None)

    temp_t = torch.tensor([w.temperature], dtype=torch.float32, device=dev)
    samp_out = [(torch.empty((R,), dtype=torch.float32, device=dev),
                 torch.empty((R,), dtype=torch.int64, device=dev)) for R in rows_l]
    flush = None

    def one_sampled(sp):
        cur = None
        for level in range(w.levels):
            smp, nd = samp_out[level]
            L.check(lib.vtnk_fused_linear_constrained_node_transition_sampling_ix(
                lins[level], L.ptr(cur), csr, dw.trie.layer_max_branches[level], w.seed,
                temp_t.data_ptr(), idxs[level], None, None, smp.data_ptr(), nd.data_ptr(), sp))
            cur = nd
        return cur

    def step_launch(level, cur, sp):
        b = bufs[level]
        L.check(lib.vtnk_beam_step(lins[level], L.ptr(cur), csr,
                                   dw.trie.layer_max_branches[level], w.topk,
                                   idxs[level], b["tok"].data_ptr(),
                                   b["logit"].data_ptr(), b["node"].data_ptr(),
                                   b["lse"].data_ptr(), sp))

    def merge_launch(level, prev_logp, prev_ids, sp):
        b = bufs[level]
        L.check(lib.vtnk_beam_merge(level, Bq, k, w.topk, b["tok"].data_ptr(),
                                    b["logit"].data_ptr(), b["node"].data_ptr(),
                                    b["lse"].data_ptr(), L.ptr(prev_logp), L.ptr(prev_ids),
                                    b["ids"].data_ptr(), b["logp"].data_ptr(),
                                    b["nxt"].data_ptr(), b["parent"].data_ptr(), sp))

    def levels_search(sp):
        """The search level by level (step + merge launches); fills every
        level's buffers (node arrays for the cost model, per-level graphs)."""
        cur = prev_logp = prev_ids = None
        for level in range(w.levels):
            b = bufs[level]
            step_launch(level, cur, sp)
            merge_launch(level, prev_logp, prev_ids, sp)
            cur, prev_logp, prev_ids = b["nxt"], b["logp"], b["ids"]

    # the timed search: the library's fused search entry point
    # (vtnk_beam_search: level 0's beams straight from the step kernel, then
    # step + merge per level), writing into this rank's result record
    keep: list = []
    search = None
    if not w.sampling:
        search = _search_struct(dw.hidden, dw.weight, None, dw.trie, k, w.topk, True, keep)
        ws = torch.empty((lib.vtnk_beam_search_workspace_bytes(search),), dtype=torch.uint8,
                         device=dev)

    def one_search(sp=None, gather=True):
        sp = sptr if sp is None else sp
        if w.sampling:
            return one_sampled(sp)
        L.check(lib.vtnk_beam_search(search, ws.data_ptr(), ws.numel(), rec.ids.data_ptr(),
                                     rec.logp.data_ptr(), rec.node.data_ptr(), sp))
        if world > 1 and gather:
            rec.gather(out=gather_buf)

    # warm-up (also records the per-level node arrays for the cost model); the
    # clock sampler starts before the last warm-up searches so that it is
    # running when the timed region begins
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = vis.split(",")[local] if vis and vis.split(",")[local].strip().isdigit() else local
    clocks = ClockSampler(int(phys))
    n_warm = max(3, args.warmup)
    if not w.sampling:
        levels_search(sptr)
        torch.cuda.synchronize(dev)
        curs = [None] + [bufs[l]["nxt"].clone() for l in range(w.levels - 1)]
    for i in range(n_warm):
        if i == n_warm - 2:
            torch.cuda.synchronize(dev)
            clocks.start()
            time.sleep(0.3)
        one_search()
    torch.cuda.synchronize(dev)
    if w.sampling:
        curs = [None] + [samp_out[l][1].clone() for l in range(w.levels - 1)]
    costs = level_costs(w, dw, curs, wins)

    # One search (every level's step and merge) captured as a CUDA graph and
    # replayed: the timed loop measures the device, not the host's launch
    # rate.  Per-level kernel times come from graphs of each launch alone.
    # Workloads whose inputs fit in L2 get a 256 MB write between timed
    # replays (timed with its own events and subtracted).
    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn(torch.cuda.current_stream(dev).cuda_stream)
        return g

    def flush_needed():
        return sum(h.numel() * h.element_size() for h in dw.hidden) < (256 << 20)

    need_flush = flush_needed()
    workload_cfg["l2"] = (
        "a search's hidden states fit in L2: a 256 MB buffer is written before every timed "
        "replay (its time subtracted)" if need_flush else
        "inputs larger than L2 (hidden states >= 0.47 GB per level), no flush")
    workload_cfg["timing"] = ("one search captured as a CUDA graph and replayed; per-level "
                              "times from graphs of each launch")
    if need_flush and flush is None:
        flush = torch.empty((256 << 20,), dtype=torch.uint8, device=dev)
    g_search = capture(lambda sp: one_search(sp=sp, gather=False))
    g_step, g_merge = [], []
    for level in range(w.levels):
        cur_l = None if level == 0 else curs[level]
        if w.sampling:
            g_step.append(capture(lambda sp, l=level, c=cur_l: L.check(
                lib.vtnk_fused_linear_constrained_node_transition_sampling_ix(
                    lins[l], L.ptr(c), csr, dw.trie.layer_max_branches[l], w.seed,
                    temp_t.data_ptr(), idxs[l], None, None, samp_out[l][0].data_ptr(),
                    samp_out[l][1].data_ptr(), sp))))
            g_merge.append(None)
        else:
            g_step.append(capture(lambda sp, l=level, c=cur_l: step_launch(l, c, sp)))
            prev = (None, None) if level == 0 else (bufs[level - 1]["logp"], bufs[level - 1]["ids"])
            g_merge.append(capture(lambda sp, l=level, pv=prev: merge_launch(l, pv[0], pv[1], sp)))
    torch.cuda.synchronize(dev)

    def replay_timed(g, n):
        """Mean device ms of n replays of g (flushing L2 before each when needed)."""
        evs = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(2)) for _ in range(n)]
        for e0, e1 in evs:
            if need_flush:
                flush.fill_(1)
            e0.record(stream)
            g.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        return statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)

    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    fev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(2))
           for _ in range(args.steps)]
    t_start.record(stream)
    for s_ in range(args.steps):
        if need_flush:
            fev[s_][0].record(stream)
            flush.fill_(1)
            fev[s_][1].record(stream)
        g_search.replay()
        if world > 1 and not w.sampling:
            rec.gather(out=gather_buf)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms_total = t_start.elapsed_time(t_end)
    if need_flush:
        ms_total -= sum(f[0].elapsed_time(f[1]) for f in fev)
    n_lvl = max(3, min(args.steps, 30))
    lvl_ms = [replay_timed(g, n_lvl) for g in g_step]
    merge_ms = [0.0 if g is None else replay_timed(g, n_lvl) for g in g_merge]
    t = torch.tensor([ms_total], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    rows_per_rank = sum(rows_l)
    value = rows_per_rank * world / (ms_per_step / 1e3)

    # roofline of the step kernel (all levels): algorithmic bytes / event time
    hbm_peak, tc_peak, peak_kind = _peaks()
    tot_bytes = sum(c[0] for c in costs)
    tot_flops = sum(c[1] for c in costs)
    t_step = sum(lvl_ms) / 1e3
    t_hbm = tot_bytes / (hbm_peak * 1e9)
    t_tc = tot_flops / (tc_peak * 1e12)
    if t_hbm >= t_tc:
        roof = {"bound": "hbm", "achieved": tot_bytes / t_step / 1e9, "peak": hbm_peak,
                "unit": "GB/s"}
    else:
        roof = {"bound": "tensor", "achieved": tot_flops / t_step / 1e12, "peak": tc_peak,
                "unit": "TFLOP/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    # DRAM bytes per hidden-state row of the step kernel, from the committed ncu
    # capture (profiles/tc_beam_step_cfg5.md: 611.1 MB for 81,920 rows at level
    # 1), scaled to this search's rows; null for other workloads
    roof["traffic"] = (round(7460.0 * sum(rows_l)) if args.workload == "cfg5" else None)
    roof["traffic_note"] = "scaled from a level-1 ncu capture (profiles/tc_beam_step_cfg5.md)"
    roof["peak_kind"] = f"{peak_kind} (MEASURED_PEAKS.json burst figures)"
    roof["kernel"] = "vtnk beam-step kernel, all levels of one search"
    roof["tensor_frac"] = (tot_flops / t_step / 1e12) / tc_peak
    roof["hbm_frac"] = (tot_bytes / t_step / 1e9) / hbm_peak
    roof["per_level_ms"] = [round(x, 4) for x in lvl_ms]
    roof["merge_ms"] = [round(x, 4) for x in merge_ms]
    if not w.sampling:
        roof["merge_note"] = ("the timed search fuses level 0's merge into its step kernel; "
                              "merge_ms[0] is the stand-alone merge kernel")
    roof["per_level_alg_bytes"] = [c[0] for c in costs]
    roof["per_level_alg_flops"] = [c[1] for c in costs]
    roof["roofline_ms"] = round(max(t_hbm, t_tc) * 1e3, 4)

    # end to end through the public API, hidden states in pinned host memory
    e2e = None
    if args.e2e_steps > 0:
        host = [h.cpu().pin_memory() for h in dw.hidden]
        if w.sampling:
            outs = (torch.empty((Bq, w.levels), dtype=torch.int64, pin_memory=True),
                    torch.empty((Bq,), dtype=torch.int64, pin_memory=True))

            def e2e_call():
                dev_h = [h.to(dev, non_blocking=True) for h in host]
                tok, node = constrained_sampling_search(dev_h, dw.weight, dw.trie, w.seed,
                                                        temp_t)
                outs[0].copy_(tok, non_blocking=True)
                outs[1].copy_(node, non_blocking=True)
        else:
            outs = (torch.empty((Bq, k, w.levels), dtype=torch.int64, pin_memory=True),
                    torch.empty((Bq * k,), dtype=torch.float32, pin_memory=True),
                    torch.empty((Bq * k,), dtype=torch.int64, pin_memory=True))

            def e2e_call():
                constrained_beam_search_from_host(host, dw.weight, dw.trie, cfg, out=outs)
        e2e_call()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_call()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        te = torch.tensor([e0.elapsed_time(e1) / args.e2e_steps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": rows_per_rank * world / (float(te.item()) / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int(sum(h.numel() * h.element_size() for h in host)),
               "d2h_bytes_per_step": int(sum(o.numel() * o.element_size() for o in outs)),
               "ms_per_step": float(te.item())}
        del host

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = CpuBaseline(w)
        nq = args.cpu_queries or 384
        dt = base.run(nq, 1)
        cpu = {"value": base.rows(nq) / dt, "unit": UNIT, "cores": 1, "kind": "port",
               "sample": f"queries 0..{nq - 1} of {args.workload}, all {w.levels} levels "
                         f"({base.rows(nq)} rows, {dt:.1f} s), fp32 numpy restatement of the "
                         f"reference's sparse path, one thread"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16" if w.dtype == "bf16" else "f32",
                "data": "synthetic (seeded catalog, N(0,0.02) head, N(0,1) hidden states)",
                "config": workload_cfg, "clocks": clk, "roofline": roof,
                "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": args.steps * (w.levels if w.sampling else 2 * w.levels - 1)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
