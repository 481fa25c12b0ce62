"""Benchmark: full constrained beam search throughput (seq*beams/s) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg5] [--impl b200|reference]

A step = one full L-level constrained beam search over this rank's shard of
the workload (config 5 by default: 16M-item catalog, H=3584, bf16, batch
65,536 x 10 beams, top-k 10; `--workload cfg4` is the Gumbel-max sampled
search), plus -- for N > 1 -- the all-gather of every rank's results (over
peer memory by default: one push + flag-barrier kernel; `--gather nccl` uses
NCCL).  Two searches are in flight on two streams, each with its own
workspace and result record (`--no-pipeline`: one at a time).
Inputs (trie, head rows, per-level hidden states) are resident in HBM before
timing.  One search is captured as a CUDA graph and replayed K times after W
warm-ups, timed with CUDA events on the launching stream.  At config 5 the
hidden states (10 GB at N=1) exceed the 126 MB L2; smaller workloads get a
256 MB write before every timed replay (timed separately and subtracted).
value = (sum over levels of rows) * N / (max over ranks of the device time
per step).

Outside the timed region the line also carries:
* `parity`: a strided sample of queries of the timed search (after the
  all-gather at N > 1: queries of every rank) against the CPU oracle;
* `e2e`: the same search through the public API with the hidden states in
  pinned host memory (host->device copies overlapped with compute, the
  all-gather at N > 1 and the device->host copy of the results inside);
* `cpu_baseline` (N = 1): the reference's sparse-PyTorch path (all host
  threads) and its CPU trie path (one thread) on a fixed query sample;
* `other_configs` (N = 1): configs 2-4 and the reference microbenchmark's
  largest op shapes, each timed the same way.

`--impl reference` times the reference's CPU implementation (its sparse-PyTorch
path, restated in oracle/cpu_paths.py -- the reference is Python and is not
installed on the GPU box) on a fixed query sample with all host threads.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "constrained beam-step seq*beams/s (full L-level search)"
UNIT = "seq*beams/s"

# Fixed CPU-baseline samples (queries, all levels) per workload.
CPU_QUERIES = {"cfg1": 4, "cfg2": 64, "cfg3": 16, "cfg4": 256, "cfg5": 64}
# DRAM bytes (read + write) per hidden-state row of the step kernel, per
# level, from the committed small-case ncu capture of all three levels
# (profiles/tc_beam_step_cfg5.md: batch 8192, dram__bytes_read/write.sum);
# scaled by the rows of a full-size launch.
TRAFFIC_PER_ROW = {"cfg5": (7430.0, 7424.7, 7527.4)}


def _peaks(sustained: bool = False):
    """(HBM GB/s, dense bf16 TFLOP/s, kind).  ``sustained``: the bf16 figure of
    a seconds-long GEMM loop under the board's power cap, the denominator for
    a kernel timed inside a long run (the step kernel draws the 1 kW cap and
    runs at ~1.3 GHz there); else the burst figure."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        tc = d.get("bf16_tflops_sustained") if sustained else None
        return d["hbm_gbs"], tc or d["bf16_tflops"], "measured"
    return 6650.0, 1400.0 if sustained else 1590.0, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks, power and throttle reasons.

    Every sample carries nvidia-smi's own wall-clock timestamp, so a summary
    can be restricted to a host-marked region (``mark``): the timed region
    and the per-level breakdown are summarised separately.  A long run of
    this step kernel draws the board's 1 kW limit and ``sw_power_cap`` lowers
    the SM clock (to ~1.3 GHz); the summaries say so instead of a median
    over idle samples."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None
        self.marks: dict[str, list[float]] = {}

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

    def mark(self, region: str, begin: bool):
        """Host wall-clock bounds of a region (after a device synchronise)."""
        self.marks.setdefault(region, [0.0, 0.0])[0 if begin else 1] = time.time()

    def _samples(self):
        out = []
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = time.mktime(time.strptime(f[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                ts += float("0." + f[0].split(".")[1]) if "." in f[0] else 0.0
                sm, smax, pw = float(f[2]), float(f[3]), float(f[4])
            except (ValueError, IndexError):
                continue
            rs = {n for n, v in zip(self.NAMES, f[6:10]) if v.lower() == "active"}
            out.append((ts, sm, smax, pw, rs))
        return out

    def stop(self) -> None:
        if self.proc is None:
            return
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)

    def summary(self, region: str | None = None) -> dict:
        """Median SM clock / power and the reasons seen inside ``region``
        (all samples when None, or when the region caught no sample)."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        smp = self._samples()
        sel = smp
        if region in self.marks:
            t0, t1 = self.marks[region]
            inside = [x for x in smp if t0 - 0.05 <= x[0] <= t1 + 0.05]
            sel = inside or sel
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = set().union(*(x[4] for x in sel))
        return {"sm_mhz": statistics.median(x[1] for x in sel),
                "sm_min_mhz": min(x[1] for x in sel),
                "sm_max_mhz": max(x[2] for x in sel),
                "power_w_median": statistics.median(x[3] for x in sel),
                "reasons": sorted(reasons), "samples": len(sel)}

    def clock_at(self, t: float) -> float | None:
        """SM clock of the sample nearest to host time ``t``."""
        smp = self._samples()
        if not smp:
            return None
        return min(smp, key=lambda x: abs(x[0] - t))[1]


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


# --------------------------------------------------------------------------- CPU baselines
class CpuSample:
    """Host inputs of a fixed query sample of workload ``w`` for the CPU
    baselines (the reference's sparse-PyTorch and CPU trie paths, restated in
    oracle/cpu_paths.py; the Gumbel-max sampled workload uses the oracle's
    sampling op, which is the reference's sparse path plus Gumbel noise)."""

    def __init__(self, w, nq: int):
        from oracle import cpu_paths as C
        from oracle import vtnk_oracle as O
        from rectokens_b200 import synthetic as S

        self.w, self.O, self.C, self.nq = w, O, C, nq
        tok = S.to_tokens(w.make_catalog(), w.codes)
        self.rp, self.cv, self.lmb, _, _ = O.build_sorted_csr(tok, w.vocab, 1)
        self.W = (S.head_f32(w.seed, w.vocab, w.hidden) if w.dtype == "f32"
                  else S.bf16_bits_to_f32(S.head_bits(w.seed, w.vocab, w.hidden)))
        self.hidden = []
        for level in range(w.levels):
            rows = nq if level == 0 else nq * w.beams
            self.hidden.append(S.hidden_f32(w.seed, level, 0, rows, w.hidden) if w.dtype == "f32"
                               else S.bf16_bits_to_f32(S.hidden_bits(w.seed, level, 0, rows,
                                                                     w.hidden)))
        self.ptrie = None

    def rows(self) -> int:
        return self.nq * (1 + self.w.beams * (self.w.levels - 1))

    def sparse(self, threads: int) -> float:
        """Seconds of one search of the sample through the sparse path."""
        import torch

        torch.set_num_threads(threads)
        w = self.w
        if w.sampling:
            t0 = time.perf_counter()
            cur = np.zeros(self.nq, dtype=np.int64)
            for level, a in enumerate(self.hidden):
                mb = self.lmb[level]
                noise = self.O.gumbel_noise(w.seed, a.shape[0], mb)
                nn, _, smp, score = self.O.fused_sampling(a, self.W.T, None, self.rp, self.cv,
                                                          cur, mb, noise, w.temperature,
                                                          acc=np.float32)
                best = np.argmax(score, axis=1)
                cur = np.where(smp >= 0, nn[np.arange(nn.shape[0]), best], -1)
            return time.perf_counter() - t0
        hid = [torch.from_numpy(h) for h in self.hidden]
        Wt, rp, cv = torch.from_numpy(self.W), torch.from_numpy(self.rp), torch.from_numpy(self.cv)
        t0 = time.perf_counter()
        self.C.sparse_path_search(hid, Wt, rp, cv, self.lmb, self.nq, w.beams, w.topk)
        return time.perf_counter() - t0

    def trie(self) -> float:
        """Seconds of one search of the sample through the CPU trie path (one
        thread; the pointer trie's visited nodes are built before timing)."""
        w = self.w
        if self.ptrie is None:
            self.ptrie = self.C.PointerTrie(self.rp, self.cv)
            trace: list = []
            self.O.beam_search(self.hidden, self.W, self.rp, self.cv, self.lmb, self.nq, w.beams,
                               w.topk, acc=np.float32, trace=trace)
            for t in trace:
                for n in np.unique(t["cur"]):
                    self.ptrie.add(int(n))
        t0 = time.perf_counter()
        self.C.trie_path_search(self.hidden, self.W, self.ptrie, self.lmb, self.nq, w.beams,
                                w.topk)
        return time.perf_counter() - t0


def cpu_baseline(w, name, rate_only=False):
    nq = min(CPU_QUERIES.get(name, 64), w.batch)
    cs = CpuSample(w, nq)
    threads = os.cpu_count() or 1
    cs.sparse(threads)  # warm-up (thread pool, allocator)
    dt = min(cs.sparse(threads) for _ in range(2))
    out = {"value": cs.rows() / dt, "unit": UNIT, "cores": threads, "kind": "port",
           "sample": f"queries 0..{nq - 1} of {name}, all {w.levels} levels ({cs.rows()} rows, "
                     f"{dt:.2f} s per search, best of 2), the reference's sparse-PyTorch path "
                     f"(fp32, torch eager on {threads} threads) driven by decode_one_step's "
                     f"route-A merge"}
    if not w.sampling and not rate_only:
        tt = cs.trie()
        out["trie_path"] = {"value": cs.rows() / tt, "unit": UNIT, "cores": 1,
                            "sample": f"the same {nq} queries through the reference's pointer "
                                      f"Trie walked row by row, fp32 dot products "
                                      f"({tt:.2f} s)"}
    return out


def reference_arm(args, w, name, workload_cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    nq = min(CPU_QUERIES.get(name, 64), w.batch)
    cs = CpuSample(w, nq)
    threads = os.cpu_count() or 1
    for _ in range(max(1, args.warmup)):
        cs.sparse(threads)
    times = [cs.sparse(threads) for _ in range(args.steps)]
    rate = cs.rows() * len(times) / sum(times)
    sample = (f"a fixed sample of {nq} queries of {name} (all {w.levels} levels, {cs.rows()} "
              f"rows) per step, {statistics.mean(times):.2f} s per step; the reference's "
              f"sparse-PyTorch path, fp32 torch eager on {threads} threads")
    line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.mean(times),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 (bf16 inputs upcast, as the reference's CPU path)",
            "data": "synthetic (seeded catalog / head / hidden states)", "config": workload_cfg,
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- one workload
def run_workload(args, w, name, dev, rank, world, extras=False):
    """Times the search of workload ``w`` on this rank's shard; returns the
    fields of the bench line (rank 0) or None."""
    import torch
    import torch.distributed as dist

    from rectokens_b200 import _lib as L
    from rectokens_b200 import synthetic as S
    from rectokens_b200 import workload as WL
    from rectokens_b200.decoding.beam_search import (
        _search_struct,
        child_index,
        constrained_beam_search_from_host,
        constrained_sampling_search,
        level_windows,
    )
    from rectokens_b200.distributed import ResultRecord, shard_queries
    from rectokens_b200.schemas import GenerationConfig
    from oracle.parity import check_sampling, check_search, parity_sample

    steps, warm = (args.steps, args.warmup) if not extras else (20, 3)
    cfg = GenerationConfig(steps=w.levels, k=w.beams, beam_size=w.topk, temperature=0.0)
    dw = WL.make_device_workload(w, dev, shard=rank, n_shards=world)
    wins = level_windows(dw.trie)
    idxs = [child_index(dw.trie, l) for l in range(w.levels)]
    Bq, k = dw.batch, w.beams
    q0, _ = shard_queries(w.batch, rank, world)

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
    # the search writes its results straight into this rank's packed record,
    # which one all-gather concatenates across ranks
    rec = ResultRecord(Bq * k, w.levels, dev)
    gather_buf = (torch.empty((world * rec.nbytes,), dtype=torch.uint8, device=dev)
                  if world > 1 else None)
    # N > 1: the results' all-gather -- over peer memory (one push + flag
    # barrier kernel, int32 ids / nodes) or NCCL (--gather nccl)
    pgather = None
    if world > 1 and not w.sampling and args.gather == "peer":
        from rectokens_b200.distributed import PeerGather

        pgather = PeerGather(Bq * k, w.levels, dev)

    def do_gather():
        if pgather is not None:
            pgather.push(rec.ids, rec.logp, rec.node)
        else:
            rec.gather(out=gather_buf)

    temp_t = torch.tensor([w.temperature], dtype=torch.float32, device=dev)
    samp_out = [(torch.empty((R,), dtype=torch.float32, device=dev),
                 torch.empty((R,), dtype=torch.int64, device=dev)) for R in rows_l]

    def one_sampled(sp):
        cur = None
        for level in range(w.levels):
            smp, nd = samp_out[level]
            L.check(lib.vtnk_fused_linear_constrained_node_transition_sampling_ix(
                lins[level], L.ptr(cur), csr, dw.trie.layer_max_branches[level], w.seed,
                temp_t.data_ptr(), idxs[level], None, None, smp.data_ptr(), nd.data_ptr(), sp))
            cur = nd

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
        """The search level by level (step + merge launches): fills every
        level's buffers for the cost model and the per-level graphs."""
        cur = prev_logp = prev_ids = None
        for level in range(w.levels):
            b = bufs[level]
            step_launch(level, cur, sp)
            merge_launch(level, prev_logp, prev_ids, sp)
            cur, prev_logp, prev_ids = b["nxt"], b["logp"], b["ids"]

    keep: list = []
    search = ws = None
    if not w.sampling:
        search = _search_struct(dw.hidden, dw.weight, None, dw.trie, k, w.topk, True, keep)
        ws = torch.empty((lib.vtnk_beam_search_workspace_bytes(search),), dtype=torch.uint8,
                         device=dev)

    def one_search(sp=None, r=None, wsb=None):
        sp = sptr if sp is None else sp
        r = rec if r is None else r
        wsb = ws if wsb is None else wsb
        if w.sampling:
            return one_sampled(sp)
        L.check(lib.vtnk_beam_search(search, wsb.data_ptr(), wsb.numel(), r.ids.data_ptr(),
                                     r.logp.data_ptr(), r.node.data_ptr(), sp))

    local = int(os.environ.get("LOCAL_RANK", "0"))
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = vis.split(",")[local] if vis and vis.split(",")[local].strip().isdigit() else local
    clocks = ClockSampler(int(phys))
    n_warm = max(3, warm)
    if not w.sampling:
        levels_search(sptr)
        torch.cuda.synchronize(dev)
        curs = [None] + [bufs[l]["nxt"].clone() for l in range(w.levels - 1)]
    for i in range(n_warm):
        if i == n_warm - 2 and not extras:
            torch.cuda.synchronize(dev)
            clocks.start()
            time.sleep(0.3)
        one_search()
        if world > 1 and not w.sampling:
            do_gather()
    torch.cuda.synchronize(dev)
    if w.sampling:
        curs = [None] + [samp_out[l][1].clone() for l in range(w.levels - 1)]
    costs = level_costs(w, dw, curs, wins)

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn(torch.cuda.current_stream(dev).cuda_stream)
        return g

    need_flush = sum(h.numel() * h.element_size() for h in dw.hidden) < (256 << 20)
    flush = torch.empty((256 << 20,), dtype=torch.uint8, device=dev) if need_flush else None
    l2_note = ("a search's hidden states fit in L2: a 256 MB buffer is written before every "
               "timed replay (its time subtracted)" if need_flush else
               "inputs larger than L2 (hidden states >= 0.47 GB per level), no flush")
    g_search = capture(lambda sp: one_search(sp=sp))
    # Two searches in flight (top-n workloads whose inputs exceed L2): search
    # i runs on stream i % 2 with its own workspace and result record, so one
    # search's ramp and partial last tile rounds overlap the other's kernels.
    # At N > 1 the peer all-gathers run in search order on their own stream;
    # a search reuses a record only after that record's previous gather.
    inflight = 2 if (not w.sampling and not need_flush and not args.no_pipeline
                     and (world == 1 or pgather is not None)) else 1
    if inflight == 2:
        rec2 = ResultRecord(Bq * k, w.levels, dev)
        ws2 = torch.empty_like(ws)
        g_search2 = capture(lambda sp: one_search(sp=sp, r=rec2, wsb=ws2))
        for _ in range(2):
            g_search2.replay()  # warm the second record and workspace
        s2 = torch.cuda.Stream(dev)
        gs = torch.cuda.Stream(dev) if pgather is not None else None
        ev_s = [torch.cuda.Event(), torch.cuda.Event()]
        ev_p = [torch.cuda.Event(), torch.cuda.Event()]
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

    def replay_timed(fn, n):
        """Mean device ms of n calls of fn (flushing L2 before each when needed)."""
        evs = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(2)) for _ in range(n)]
        for e0, e1 in evs:
            if need_flush:
                flush.fill_(1)
            e0.record(stream)
            fn()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        return statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)

    # ---------------------------------------------------------------- timed region
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.mark("timed", True)
    fev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(2)) for _ in range(steps)]
    t_start.record(stream)
    for s_ in range(steps):
        if need_flush:
            fev[s_][0].record(stream)
            flush.fill_(1)
            fev[s_][1].record(stream)
        if inflight == 2:
            i = s_ & 1
            st = (stream, s2)[i]
            if s_ == 1:
                s2.wait_stream(stream)  # after t_start
            if s_ >= 2 and gs is not None:
                st.wait_event(ev_p[i])  # this record's previous gather is done
            with torch.cuda.stream(st):
                (g_search, g_search2)[i].replay()
            if gs is not None:
                ev_s[i].record(st)
                gs.wait_event(ev_s[i])
                r = (rec, rec2)[i]
                pgather.push(r.ids, r.logp, r.node, stream=gs.cuda_stream)
                ev_p[i].record(gs)
            continue
        g_search.replay()
        if world > 1 and not w.sampling:
            do_gather()
    if inflight == 2:  # every search and gather inside the timed region
        stream.wait_stream(s2)
        if gs is not None:
            stream.wait_stream(gs)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    clocks.mark("timed", False)
    if world > 1:
        dist.barrier()
    ms_total = t_start.elapsed_time(t_end)
    if need_flush:
        ms_total -= sum(f[0].elapsed_time(f[1]) for f in fev)
    # ---------------------------------------------------------------- breakdown
    n_lvl = max(3, min(steps, 30))
    clocks.mark("breakdown", True)
    lvl_ms = [replay_timed(g.replay, n_lvl) for g in g_step]
    merge_ms = [0.0 if g is None else replay_timed(g.replay, n_lvl) for g in g_merge]
    clocks.mark("breakdown", False)
    # Sustained replay of the largest level's step kernel: launch times binned
    # by the SM clock sampled at the time (the board's power cap lowers it).
    sustain = None
    if not extras and args.sustain > 0 and rank == 0:
        lv = max(range(w.levels), key=lambda l: rows_l[l])
        batches = []
        t_end_s = time.time() + args.sustain
        while time.time() < t_end_s:
            b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b0.record(stream)
            for _ in range(5):
                g_step[lv].replay()
            b1.record(stream)
            torch.cuda.synchronize(dev)
            batches.append((time.time(), b0.elapsed_time(b1) / 5))
        time.sleep(1.0)  # idle: the clock recovers
        for _ in range(3):
            b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b0.record(stream)
            g_step[lv].replay()
            b1.record(stream)
            torch.cuda.synchronize(dev)
            batches.append((time.time(), b0.elapsed_time(b1)))
    if not extras:
        clocks.stop()
        if sustain is None and args.sustain > 0 and rank == 0:
            bins: dict = {}
            for tb, ms in batches:
                mhz = clocks.clock_at(tb)
                if mhz is None:
                    continue
                key = int(mhz // 100) * 100
                bins.setdefault(key, []).append(ms)
            sustain = {"level": lv, "seconds": args.sustain,
                       "by_sm_mhz": [{"sm_mhz": f"{k}-{k + 99}", "launches": 5 * len(v),
                                      "ms_median": round(statistics.median(v), 4)}
                                     for k, v in sorted(bins.items())],
                       "note": "the level's step kernel replayed back to back; each 5-launch "
                               "batch binned by the nvidia-smi SM-clock sample nearest to it "
                               "(the last entries after 1 s idle)"}
    clk = None
    if not extras:
        clk = clocks.summary("timed")
        clk["breakdown"] = clocks.summary("breakdown")
    search_ms = replay_timed(g_search.replay, n_lvl)
    gather_ms = None
    if world > 1 and not w.sampling:
        dist.barrier()
        gather_ms = replay_timed(do_gather, n_lvl)
    t = torch.tensor([ms_total, search_ms, gather_ms or 0.0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t[0].item()) / steps
    rows_per_rank = sum(rows_l)
    value = rows_per_rank * world / (ms_per_step / 1e3)

    hbm_peak, tc_peak, peak_kind = _peaks(sustained=True)
    tc_burst = _peaks()[1]
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
    tpr = TRAFFIC_PER_ROW.get(name)
    roof["traffic"] = (round(sum(tpr[l] * rows_l[l] for l in range(w.levels)))
                       if tpr and len(tpr) >= w.levels else None)
    roof["traffic_note"] = ("per-level DRAM bytes per row from a small-case ncu capture of "
                            "all three levels (profiles/tc_beam_step_cfg5.md), scaled by "
                            "this search's rows")
    roof["peak_kind"] = (f"{peak_kind}: HBM copy bandwidth and the sustained bf16 GEMM figure "
                         "(the kernels are timed in back-to-back replays, where the board's "
                         "power cap holds the SM clock near 1.3 GHz; see clocks.breakdown)")
    roof["tensor_frac_burst"] = (tot_flops / t_step / 1e12) / tc_burst
    roof["kernel"] = "vtnk beam-step kernel, all levels of one search"
    roof["tensor_frac"] = (tot_flops / t_step / 1e12) / tc_peak
    roof["hbm_frac"] = (tot_bytes / t_step / 1e9) / hbm_peak
    roof["per_level_ms"] = [round(x, 4) for x in lvl_ms]
    roof["per_level_roofline_ms"] = [round(max(c[0] / (hbm_peak * 1e9), c[1] / (tc_peak * 1e12))
                                           * 1e3, 4) for c in costs]
    roof["merge_ms"] = [round(x, 4) for x in merge_ms]
    if not w.sampling:
        roof["merge_note"] = ("the timed search fuses level 0's merge into its step kernel; "
                              "merge_ms[0] is the stand-alone merge kernel")
    roof["per_level_alg_bytes"] = [c[0] for c in costs]
    roof["per_level_alg_flops"] = [c[1] for c in costs]
    roof["roofline_ms"] = round(max(t_hbm, t_tc) * 1e3, 4)
    breakdown = {"search_ms": round(float(t[1].item()), 4),
                 "gather_ms": round(float(t[2].item()), 4) if gather_ms is not None else None,
                 "gather": args.gather if world > 1 else None,
                 "searches_in_flight": inflight,
                 "step_ms": [round(x, 4) for x in lvl_ms],
                 "merge_ms": [round(x, 4) for x in merge_ms[1:]] if not w.sampling else []}

    # ---------------------------------------------------------------- parity (not timed)
    parity = None
    if not args.no_parity:
        torch.cuda.synchronize(dev)
        if world > 1 and not w.sampling:
            if pgather is not None:
                do_gather()
                g_ids, g_logp, g_node, pstatus = pgather.result()
                if pstatus:
                    raise RuntimeError(f"peer gather status {pstatus}")
            else:
                g_ids, g_logp, g_node = rec.gather(out=gather_buf)
            all_ids = g_ids.reshape(w.batch, k, w.levels).cpu().numpy()
            all_logp = g_logp.reshape(-1).cpu().numpy()
            all_node = g_node.reshape(-1).cpu().numpy()
        elif not w.sampling:
            all_ids = rec.ids.view(Bq, k, w.levels).cpu().numpy()
            all_logp = rec.logp.cpu().numpy()
            all_node = rec.node.cpu().numpy()
        if rank == 0:
            rp = dw.trie.row_ptrs.cpu().numpy()
            cv = dw.trie.stacked_cols_vals.cpu().numpy()
            W64 = dw.weight.double().cpu().numpy()
            lmb = dw.trie.layer_max_branches
            if w.sampling:
                from rectokens_b200.ops._vtnk_ops import gumbel_noise

                qs = parity_sample(Bq, 256)
                tok = torch.stack([samp_out[l][0] for l in range(w.levels)], 1)
                tok = tok.cpu().numpy().astype(np.int64)[qs]
                node = samp_out[-1][1].cpu().numpy()[qs]
                nmax = int(qs.max()) + 1

                def noise_fn(level, queries, mb):
                    return gumbel_noise(w.seed, nmax, mb, dev).cpu().numpy()[queries]

                parity = check_sampling(w, rp, cv, lmb, W64, qs, tok, node, noise_fn, q0)
                parity["sample"] = f"{len(qs)} strided sequences of this rank's shard"
            else:
                qs = parity_sample(w.batch if world > 1 else Bq)
                sel = (qs[:, None] * k + np.arange(k)[None, :]).reshape(-1)
                parity = check_search(w, rp, cv, lmb, W64, qs + (0 if world > 1 else q0),
                                      all_ids[qs], all_logp[sel], all_node[sel])
                parity["sample"] = (f"{len(qs)} strided queries of the gathered {world}-rank "
                                    "result" if world > 1 else
                                    f"{len(qs)} strided queries of the timed search")
        if world > 1:
            dist.barrier()

    # ---------------------------------------------------------------- e2e
    e2e = None
    e2e_steps = args.e2e_steps if not extras else 2
    if e2e_steps > 0:
        host = [h.cpu().pin_memory() for h in dw.hidden]
        if w.sampling:
            outs = (torch.empty((Bq, w.levels), dtype=torch.int64, pin_memory=True),
                    torch.empty((Bq,), dtype=torch.int64, pin_memory=True))

            def e2e_call():
                dev_h = [h.to(dev, non_blocking=True) for h in host]
                tk, nd = constrained_sampling_search(dev_h, dw.weight, dw.trie, w.seed, temp_t)
                outs[0].copy_(tk, non_blocking=True)
                outs[1].copy_(nd, non_blocking=True)
        elif world == 1:
            outs = (torch.empty((Bq, k, w.levels), dtype=torch.int64, pin_memory=True),
                    torch.empty((Bq * k,), dtype=torch.float32, pin_memory=True),
                    torch.empty((Bq * k,), dtype=torch.int64, pin_memory=True))

            def e2e_call():
                constrained_beam_search_from_host(host, dw.weight, dw.trie, cfg, out=outs)
        else:
            # the search on this rank's shard, its results packed and
            # all-gathered, the gathered results read back by rank 0
            e2e_rec = ResultRecord(Bq * k, w.levels, dev)
            if pgather is not None:
                outs = (torch.empty((world, Bq * k, w.levels), dtype=torch.int32,
                                    pin_memory=True),
                        torch.empty((world, Bq * k), dtype=torch.float32, pin_memory=True),
                        torch.empty((world, Bq * k), dtype=torch.int32, pin_memory=True))
            else:
                outs = (torch.empty((world * rec.nbytes,), dtype=torch.uint8, pin_memory=True),)
                e2e_gather = torch.empty_like(gather_buf)

            def e2e_call():
                r = constrained_beam_search_from_host(host, dw.weight, dw.trie, cfg,
                                                      device_out=True)
                if pgather is not None:
                    pgather.push(r.generated_ids.view(Bq * k, w.levels), r.log_probas,
                                 r.cur_node)
                    if rank == 0:
                        for o, x in zip(outs, pgather.result()[:3]):
                            o.copy_(x, non_blocking=True)
                else:
                    e2e_rec.ids.copy_(r.generated_ids.view(Bq * k, w.levels))
                    e2e_rec.logp.copy_(r.log_probas)
                    e2e_rec.node.copy_(r.cur_node)
                    e2e_rec.gather(out=e2e_gather)
                    if rank == 0:
                        outs[0].copy_(e2e_gather, non_blocking=True)
                torch.cuda.current_stream(dev).synchronize()
        e2e_call()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_call()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        te = torch.tensor([e0.elapsed_time(e1) / e2e_steps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": rows_per_rank * world / (float(te.item()) / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int(sum(h.numel() * h.element_size() for h in host)) * world,
               "d2h_bytes_per_step": int(sum(o.numel() * o.element_size() for o in outs)),
               "ms_per_step": float(te.item()),
               "path": ("public API: constrained_beam_search_from_host per level (H2D of level "
                        "l+1 overlapped with level l), " +
                        (f"results all-gathered ({args.gather}) and read back by rank 0"
                         if world > 1 else "results read back to pinned host memory"))}
        del host

    launches = steps * (w.levels if w.sampling else 2 * w.levels - 1)
    if sustain is not None:
        roof["sustained"] = sustain
    return dict(value=value, ms_per_step=ms_per_step, steps=steps, warmup=warm, clocks=clk,
                roofline=roof, e2e=e2e, parity=parity, breakdown=breakdown,
                gpu_launches=launches, l2=l2_note, dtype="bf16" if w.dtype == "bf16" else "f32")


# --------------------------------------------------------------------------- op microbenchmarks
def op_bench(dev):
    """The reference microbenchmark's largest shape (B=4096, N=150,000,
    max_branches=1,500, K=512, fp32, every row at the root;
    examples/scripts/benchmark/benchmark_vtnk.py:30,43-51,108,120-170) through
    the drop-in ops, timed like triton's do_bench (25 ms-ish warm-up, 100
    reps, CUDA events), beside the reference's published numbers
    (out/bench_vtnk.csv:13, out/bench_fused_topk.csv:7; hardware unstated)."""
    import torch

    from rectokens_b200.ops.constrained_node_transition import (
        constrained_node_transition,
        fused_linear_constrained_node_transition,
        fused_linear_constrained_node_transition_topk,
    )
    from rectokens_b200.schemas import CompactCSRTrie, ConstraintState

    B, N, K, mb = 4096, 150_000, 512, 1500
    g = torch.Generator(device=dev).manual_seed(0)
    seqs = torch.arange(mb, dtype=torch.long).unsqueeze(1)
    trie = CompactCSRTrie.from_sorted_batch(seqs, vocab_size=N)
    trie = trie._replace(row_ptrs=trie.row_ptrs.to(dev),
                         stacked_cols_vals=trie.stacked_cols_vals.to(dev))
    a = torch.randn(B, K, device=dev, generator=g)
    weight = torch.randn(N, K, device=dev, generator=g)
    cs = ConstraintState(step=0, trie=trie, cur_node=torch.zeros(B, dtype=torch.long, device=dev))

    def bench(fn, rep=100, warm=25):
        for _ in range(warm):
            fn()
        evs = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(2)) for _ in range(rep)]
        for e0, e1 in evs:
            e0.record()
            fn()
            e1.record()
        torch.cuda.synchronize(dev)
        return statistics.median(e0.elapsed_time(e1) for e0, e1 in evs)

    out = {"shape": f"B={B}, N={N}, max_branches={mb}, K={K}, fp32, cur_node = root",
           "timing": "median of 100 reps after 25 warm-up calls, CUDA events"}
    fused_ms = bench(lambda: fused_linear_constrained_node_transition(a, weight.T, cs))
    out["fused_ms"] = round(fused_ms, 4)
    out["fused_ref_published_ms"] = 9.952
    # full corrected_logits write dominates: B*N*4 bytes + a, the 1,500 W rows
    # and the [B, max_branches] next_node / valid_idxs tables
    out["fused_hbm_frac"] = (B * N * 4 + B * K * 4 + mb * K * 4 + B * mb * 16) / (
        fused_ms / 1e3) / (_peaks()[0] * 1e9)
    logits = a @ weight.T
    mask_ms = bench(lambda: constrained_node_transition(logits, cs))
    route_ms = bench(lambda: constrained_node_transition(a @ weight.T, cs))
    out["mask_only_ms"] = round(mask_ms, 4)
    # the op writes every column and reads only the child columns of the logits
    out["mask_only_hbm_frac"] = (B * N * 4 + B * mb * 4 + B * mb * 16) / (mask_ms / 1e3) / (
        _peaks()[0] * 1e9)
    out["mask_route_ms"] = round(route_ms, 4)
    out["mask_route_note"] = "a @ W.T (cuBLAS, fp32) + the mask-only op, as the reference times it"
    out["mask_route_ref_published_ms"] = 814.527
    topk_ms = bench(lambda: fused_linear_constrained_node_transition_topk(a, weight.T, cs, 50))
    out["topk50_ms"] = round(topk_ms, 4)
    out["topk50_ref_published_ms"] = 5.755
    del logits
    return out


# --------------------------------------------------------------------------- main
def workload_config(name, w, gpus):
    return {
        "workload": (f"{name}: {w.levels}-level Gumbel-max sampled search "
                     f"(T={w.temperature}, Philox seed {w.seed}), catalog K={w.codes} "
                     f"L={w.levels}, H={w.hidden} {w.dtype} head, batch {w.batch}"
                     if w.sampling else
                     f"{name}: {w.levels}-level beam search, catalog K={w.codes} "
                     f"L={w.levels}, H={w.hidden} {w.dtype} head, batch {w.batch} x {w.beams} "
                     f"beams, top-{w.topk}"),
        "global_batch": w.batch, "beams": w.beams, "topk": w.topk, "levels": w.levels,
        "hidden": w.hidden, "rows_per_search": sum(w.rows(l) for l in range(w.levels)),
        "parallelism": f"dp{gpus}" if gpus > 1 else "single",
    }


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
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-pipeline", action="store_true",
                    help="one search in flight (default: two, on two streams)")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="N > 1: the results' all-gather over peer memory or NCCL")
    ap.add_argument("--sustain", type=float, default=3.0,
                    help="seconds of back-to-back replays of the largest level's step kernel, "
                         "binned by SM clock (0: skip)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the other configs and the op microbenchmarks (N = 1)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    from rectokens_b200 import synthetic as S

    w = S.WORKLOADS[args.workload]
    if args.batch:
        w = dataclasses.replace(w, batch=args.batch)
    workload_cfg = workload_config(args.workload, w, args.gpus)

    if args.impl == "reference":
        reference_arm(args, w, args.workload, workload_cfg)
        return

    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    r = run_workload(args, w, args.workload, dev, rank, world)
    workload_cfg["l2"] = r["l2"]
    workload_cfg["timing"] = ("one search captured as a CUDA graph and replayed; per-level "
                              "times from graphs of each launch" +
                              ("; two searches in flight on two streams (own workspace and "
                               "result record each; at N > 1 the all-gathers in order on a third "
                               "stream), every search and gather inside the timed region"
                               if r["breakdown"].get("searches_in_flight", 1) == 2 else ""))

    others = None
    if world == 1 and not args.no_extras and args.workload == "cfg5" and not args.batch:
        torch.cuda.empty_cache()
        others = {}
        for name in ("cfg2", "cfg3", "cfg4"):
            wo = S.WORKLOADS[name]
            ro = run_workload(args, wo, name, dev, 0, 1, extras=True)
            others[name] = {
                "workload": workload_config(name, wo, 1)["workload"],
                "value": ro["value"], "unit": UNIT, "ms_per_step": ro["ms_per_step"],
                "per_level_ms": ro["roofline"]["per_level_ms"],
                "per_level_roofline_ms": ro["roofline"]["per_level_roofline_ms"],
                "merge_ms": ro["roofline"]["merge_ms"],
                "roofline_frac": ro["roofline"]["frac"], "roofline_bound": ro["roofline"]["bound"],
                "roofline_ms": ro["roofline"]["roofline_ms"],
                "e2e": ro["e2e"], "parity": ro["parity"], "l2": ro["l2"]}
            torch.cuda.empty_cache()
        others["ops_reference_microbenchmark"] = op_bench(dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, args.workload)

    if rank == 0:
        line = {"metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": world,
                "steps": r["steps"], "warmup": r["warmup"], "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": r["dtype"],
                "data": "synthetic (seeded catalog, N(0,0.02) head, N(0,1) hidden states)",
                "config": workload_cfg, "clocks": r["clocks"], "roofline": r["roofline"],
                "breakdown": r["breakdown"], "parity": r["parity"],
                "cpu_baseline": cpu, "e2e": r["e2e"], "gpu_launches": r["gpu_launches"]}
        if others is not None:
            line["other_configs"] = others
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
