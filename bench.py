"""Benchmark of the speculative-decoding hot path (one JSON line on rank 0).

Workload (per GPU, weak scaling): the end-to-end draft -> verify -> accept
step of 32 sequences: hashed trigram drafting (2^20 x 8 table, Zipf(1.2)
counts) into trees of <= 64 nodes (4 at depth 1, 2 below, depth <= 5), tree
attention over 16-token KV pages with context 32768 (GQA 32/4, d=128, bf16),
the LM head [nodes, 2048] x [151936, 2048]^T (bf16, this library's tcgen05
kernel, which also writes the acceptance's chunk keys), sampling acceptance at
T=0.7 with seeded uniforms (records from those keys), and KV compaction.
Inputs are seeded synthetic tensors (no dataset exists for this path).

metric: accepted tokens/s (emitted tokens = accepted drafts + bonus, summed over
all ranks, over the max-over-ranks device time). On one GPU the line also
carries `configs`: device time per launch and roofline fraction of the kernels
of the four single-GPU configurations (greedy chain, greedy tree, sampling
against draft logits, tree attention + greedy acceptance + compaction) and of
the C5 LM head and acceptance (with the streaming acceptance over the logits
and cuBLAS's product for comparison).

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Multi-GPU: launched by torch.distributed.run, one rank per GPU. The only
collective is an all-reduce of the acceptance counters every few steps, on a
side stream, so it overlaps the compute stream.

--impl reference times the same per-GPU step on the host cores the reference's
way (its attention statements, LM head and sampler in torch, its own C++
verifier for the acceptance decisions where oracle/_ref is built). That arm
never loads liba11spec.so: it reads the seeded generators from
a11spec/workloads.py by file path, without importing the package.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "a11-llm-optimizer_b200")
sys.path[:0] = [ROOT, PKG]

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "accepted tokens/s"
UNIT = "tokens/s"
B_PER_GPU, CTX, MAX_NODES, HQ, HKV, D, HIDDEN, VOCAB, TEMP = 32, 32768, 64, 32, 4, 128, 2048, 151936, 0.7
WIDTH_ROOT, WIDTH_INNER, MAX_DEPTH = 4, 2, 5
SPARE_PAGES = 32  # per sequence: room for the context to grow by the committed tokens
LOG2_BUCKETS = 20
REDUCE_EVERY = 5  # steps between two all-reduces of the acceptance counters (multi-GPU)
STAT_NAMES = ("steps_accepted", "steps_rejected", "fallback_count", "total_draft_tokens",
              "total_steps", "emitted_tokens")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return dict(hbm=d["hbm_gbs"], tflops=d["bf16_tflops"], tflops_sus=d["bf16_tflops_sustained"],
                    src="measured")
    return dict(hbm=6650.0, tflops=1590.0, tflops_sus=1400.0, src="fallback")


def profile_traffic(kernel_key: str):
    """dram bytes per launch recorded from an ncu capture (profiles/*.md)."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for fn in sorted(os.listdir(pdir)):
        if not fn.endswith((".md", ".txt")):
            continue
        for line in open(os.path.join(pdir, fn)):
            if line.startswith(f"traffic_bytes_per_launch[{kernel_key}]:"):
                try:
                    return float(line.split(":", 1)[1].split()[0])
                except ValueError:
                    return None
    return None


def workloads_module():
    """a11spec/workloads.py loaded by file path: it needs numpy and torch only,
    so the host arms never load the CUDA library through the package."""
    spec = importlib.util.spec_from_file_location("a11spec_workloads_host",
                                                  os.path.join(PKG, "a11spec", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def workload_config(world: int) -> dict:
    """The `config` of both arms' lines (the driver compares them)."""
    return {"workload": "C5 end-to-end draft->reserve pages->verify->accept->compact->release pages, "
                        "32 seqs/GPU, context growing from 32768 by the committed tokens",
            "seqs_per_gpu": B_PER_GPU, "global_seqs": B_PER_GPU * world, "ctx": CTX, "max_nodes": MAX_NODES,
            "gqa": f"{HQ}/{HKV}", "head_dim": D, "vocab": VOCAB, "temperature": TEMP,
            "parallelism": f"request-batch dp{world}",
            "l2": "inputs larger than L2 (2.15 GB KV, 622 MB LM-head weight and 622 MB logits per step)"}


def gpu_id(dev) -> str:
    """nvidia-smi --id value of a torch device (its UUID; robust to CUDA_VISIBLE_DEVICES)."""
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev.index or 0)


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()  # the timed region starts once samples flow
            while not self.lines and time.time() - t0 < 3.0:
                time.sleep(0.01)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def device_time_us(fn, iters: int, pre=None, warmup: int = 1) -> float:
    """Mean device time of fn(i) over `iters` launches, each between its own
    pair of CUDA events on the current stream, after `warmup` untimed launches
    (fn(0)). A GPU-side spin queued first keeps the device busy while the host
    enqueues every launch, so host launch overhead never shows up as device
    time. pre(i) runs outside the events."""
    for _ in range(warmup):
        if pre is not None:
            pre(0)
        fn(0)
    torch.cuda.synchronize()
    torch.cuda._sleep(100_000_000)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for i, (a, b) in enumerate(evs):
        if pre is not None:
            pre(i)
        a.record()
        fn(i)
        b.record()
    torch.cuda.synchronize()
    return 1e3 * sum(a.elapsed_time(b) for a, b in evs) / iters


# ----------------------------------------------------------------------------- C1-C4 kernels
def measure_configs(dev, pk, c5=None) -> dict:
    """Device time per launch of the kernels of the single-GPU configurations,
    with algorithmic bytes or FLOPs and the fraction of the measured peak.
    Between timed launches the inputs rotate over copies larger than L2 in
    total (C1, C2), or a single copy already exceeds L2 (C3, C4, C5).
    c5: the C5 step's state (hidden, w_out, logits, keys, tree, uniforms)."""
    import a11spec
    from a11spec import workloads as W

    hbm = pk["hbm"]
    out = {}

    def hbm_entry(us, nbytes, launches, note):
        gbs = nbytes / (us * 1e-6) / 1e9
        return {"us_per_launch": us, "bytes_per_launch": nbytes, "achieved_gbs": gbs,
                "frac_hbm": gbs / hbm, "kernel_launches": launches, "note": note}

    if c5 is not None:
        # C5 LM head [2048, 2048] x [2048, 151936] and its acceptance, on the step's last state
        hid, w_out, logits, keys = c5["hidden"], c5["w_out"], c5["logits"], c5["keys"]
        tk, pa, nn, uni = c5["tree"]
        Bc, Nc = tk.shape
        lmws = a11spec.ops.workspace(256, dev)
        flops = 2.0 * hid.shape[0] * hid.shape[1] * w_out.shape[0]
        us = device_time_us(lambda i: a11spec.lm_head(hid, w_out, out=logits, keys=keys, ws=lmws), 10)
        tf = flops / (us * 1e-6) / 1e12
        out["C5_lm_head"] = {"us_per_launch": us, "flops_per_launch": flops, "achieved_tflops": tf,
                             "frac_tensor_burst": tf / pk["tflops"], "bound": "tensor", "kernel_launches": 1,
                             "note": "logits and the chunk keys of the acceptance (tcgen05, TMA stores)"}
        # cuBLAS on the same product, for comparison (not on the step's path): the faster of the
        # weight as stored ([vocab, hidden], F.linear) and a [hidden, vocab] copy (torch.matmul)
        us_nt = device_time_us(lambda i: torch.nn.functional.linear(hid, w_out), 4)
        w_hv = w_out.t().contiguous()
        us_nn = device_time_us(lambda i: torch.matmul(hid, w_hv, out=logits), 10)
        del w_hv
        us = min(us_nt, us_nn)
        tf = flops / (us * 1e-6) / 1e12
        out["C5_lm_head_cublas"] = {"us_per_launch": us, "achieved_tflops": tf, "frac_tensor_burst": tf / pk["tflops"],
                                    "us_weight_as_stored": us_nt, "us_weight_transposed_copy": us_nn,
                                    "note": "the same product by cuBLAS, for comparison; not on the step's path"}
        a11spec.lm_head(hid, w_out, out=logits, keys=keys, ws=lmws)  # the keys of these logits
        lg3 = logits.view(Bc, Nc, -1)
        acc = a11spec.ops.alloc_accept(a11spec.STOCH_ONEHOT, Bc, Nc, lg3.shape[2], dev)
        us = device_time_us(lambda i: a11spec.accept(a11spec.STOCH_ONEHOT, lg3, tk, pa, nn, temperature=TEMP,
                                                     uniforms=uni, out=acc), 10)
        out["C5_accept_stream"] = hbm_entry(us, lg3.numel() * 2, 2,
                                            "a11s_accept over the 622 MB of logits (record init + accept "
                                            "kernel): the pass the step replaces with the LM head's keys")
        us = device_time_us(lambda i: a11spec.accept(a11spec.STOCH_ONEHOT, lg3, tk, pa, nn, temperature=TEMP,
                                                     uniforms=uni, out=acc, keys=keys), 10)
        out["C5_accept_recorded"] = {"us_per_launch": us, "bound": "latency", "kernel_launches": 2,
                                     "mean_accept_len": float(acc.accept_len.float().mean()),
                                     "note": "records from the LM head's keys (init) + the walk; reads the "
                                             "visited rows only"}
        del acc

    # C1: greedy chain, B=1, fp32 [6, 32000]: latency-bound
    d = W.make_c1(seed=1)
    copies = 200  # 200 x 768 KB = 154 MB > L2
    lg = torch.from_numpy(d["logits"]).to(dev).expand(copies, -1, -1, -1).contiguous()
    tk, pa, nn = (torch.from_numpy(d[k]).to(dev) for k in ("tokens", "parents", "n_nodes"))
    acc = a11spec.ops.alloc_accept(a11spec.GREEDY, 1, 6, 32000, dev)
    us = device_time_us(lambda i: a11spec.accept(a11spec.GREEDY, lg[i], tk, pa, nn, out=acc), copies)
    out["C1_greedy_chain"] = {"us_per_launch": us, "bytes_per_launch": 6 * 32000 * 4, "bound": "latency",
                              "kernel_launches": 2, "accept_len": int(acc.accept_len[0]),
                              "note": "record init + accept kernel; inputs rotate over 200 copies (154 MB)"}
    del lg

    # C2: greedy complete binary tree, B=8, bf16 [8, 31, 151936], 60 % forced matches
    d = W.make_c2(seed=2)
    copies = 3  # 3 x 75 MB > L2
    lg = d["logits_bf16"].to(dev).expand(copies, -1, -1, -1).contiguous()
    tk, pa, nn = (torch.from_numpy(d[k]).to(dev) for k in ("tokens", "parents", "n_nodes"))
    acc = a11spec.ops.alloc_accept(a11spec.GREEDY, 8, 31, VOCAB, dev)
    us = device_time_us(lambda i: a11spec.accept(a11spec.GREEDY, lg[i % copies], tk, pa, nn, out=acc), 30)
    e = hbm_entry(us, 8 * 31 * VOCAB * 2, 2, "record init + accept kernel; inputs rotate over 3 copies (226 MB)")
    e["mean_accept_len"] = float(acc.accept_len.float().mean())
    out["C2_greedy_tree"] = e
    del lg

    # C3: sampling against draft logits, T=0.8, B=64, 63 drafts, fp32 p and q (4.98 GB)
    d = W.make_c3(seed=3, device=dev)
    acc = a11spec.ops.alloc_accept(a11spec.STOCH_DRAFT, 64, 64, VOCAB, dev)
    us = device_time_us(lambda i: a11spec.accept(a11spec.STOCH_DRAFT, d["p"], d["tokens"], d["parents"], d["n_nodes"],
                                                 draft_logits=d["q"], temperature=0.8, uniforms=d["uniforms"],
                                                 out=acc), 4)
    e = hbm_entry(us, 2 * 64 * 64 * VOCAB * 4, 2, "record init + accept kernel; p and q read once")
    e["mean_accept_len"] = float(acc.accept_len.float().mean())
    out["C3_draft_sampling"] = e
    del d, acc

    # C4: tree attention (ctx 4096, GQA 32/4, 64-node random trees) + greedy accept + compaction, B=32
    d = W.make_c4(seed=4, device=dev)
    B, N = 32, 64
    attn_out = torch.empty_like(d["q"])
    ws = a11spec.ops.workspace(a11spec.ops.tree_attention_workspace_bytes(B, N, HQ, HKV, D, 4096 + N), dev)
    us = device_time_us(lambda i: a11spec.tree_attention(d["q"], d["k_pool"], d["v_pool"], d["page_table"],
                                                         d["ctx_lens"], d["parents"], d["n_nodes"], out=attn_out,
                                                         ws=ws), 10)
    flops = 4.0 * B * HQ * N * (4096 + N / 2) * D
    tf = flops / (us * 1e-6) / 1e12
    out["C4_tree_attention"] = {"us_per_launch": us, "flops_per_launch": flops, "achieved_tflops": tf,
                                "frac_tensor_burst": tf / pk["tflops"], "bound": "tensor",
                                "note": "KV 273 MB + Q/O 34 MB per launch"}
    acc = a11spec.ops.alloc_accept(a11spec.GREEDY, B, N, VOCAB, dev)
    us = device_time_us(lambda i: a11spec.accept(a11spec.GREEDY, d["logits"], d["tokens"], d["parents"],
                                                 d["n_nodes"], out=acc), 10)
    e = hbm_entry(us, B * N * VOCAB * 2, 2, "record init + accept kernel; 622 MB of logits")
    e["mean_accept_len"] = float(acc.accept_len.float().mean())
    out["C4_greedy_accept"] = e
    pt0, len0 = d["page_table"].clone(), d["ctx_lens"].clone()
    freed = torch.full_like(pt0, -1)
    n_freed = torch.zeros(B, dtype=torch.int32, device=dev)
    kws = a11spec.ops.workspace(256, dev)

    def restore(i):
        d["page_table"].copy_(pt0)
        d["ctx_lens"].copy_(len0)

    us = device_time_us(lambda i: a11spec.kv_compact(d["k_pool"], d["v_pool"], d["page_table"], d["ctx_lens"],
                                                     acc.accept_len, acc.accepted_nodes, d["n_nodes"],
                                                     freed_pages=freed, n_freed=n_freed, ws=kws), 10, pre=restore)
    moved = int(acc.accept_len.sum())
    out["C4_compaction"] = {"us_per_launch": us, "bytes_per_launch": 2 * 2 * moved * HKV * D * 2,
                            "bound": "latency", "kernel_launches": 2, "rows_moved": moved,
                            "note": "K and V rows of the accepted nodes read and written once, then the "
                                    "page-table shrink"}
    del d, acc
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import a11spec
    from a11spec import workloads as W

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B = B_PER_GPU
    st = W.make_c5(seed=5 + 1000 * rank, batch=B, ctx=CTX, max_nodes=MAX_NODES, num_q_heads=HQ,
                   num_kv_heads=HKV, head_dim=D, hidden=HIDDEN, vocab=VOCAB, log2_buckets=LOG2_BUCKETS,
                   device=str(dev), temperature=TEMP, spare_pages=SPARE_PAGES)
    host_copy = None
    if world == 1 and not args.no_cpu_baseline:
        host_copy = host_state(st)  # before the step changes the page tables and lengths
    table, q, hidden = st["table"], st["q"], st["hidden"]
    # the output projection as a model stores it, [vocab, hidden] (output_w of engine/pipeline.py:470)
    w_out = st["w"].t().contiguous()
    del st["w"]
    k_pool, v_pool = st["k_pool"], st["v_pool"]
    page_table, ctx_lens = st["page_table"], st["ctx_lens"]
    # the device page allocator owns every page no context holds; each step
    # reserves the drafted tree's slots and takes back what compaction detaches
    page_table[:, (CTX + 15) // 16:] = -1
    pages = a11spec.ops.KVPagePool(k_pool.shape[0], dev)
    pages.adopt(page_table)
    last = st["last_tokens"]
    stats = torch.zeros(a11spec.STATS_LEN, dtype=torch.int64, device=dev)
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    max_kv = CTX + MAX_NODES + SPARE_PAGES * 16  # the context grows by the committed tokens
    # persistent buffers and workspaces: the step allocates nothing
    tree = (torch.empty(B, MAX_NODES, dtype=torch.int32, device=dev),
            torch.empty(B, MAX_NODES, dtype=torch.int32, device=dev),
            torch.empty(B, MAX_NODES, dtype=torch.int32, device=dev),
            torch.empty(B, dtype=torch.int32, device=dev))
    attn_out = torch.empty_like(q)
    attn_ws = a11spec.ops.workspace(a11spec.ops.tree_attention_workspace_bytes(B, MAX_NODES, HQ, HKV, D, max_kv), dev)
    # liba11spec kernels per step: n-gram expand, page reserve, tree attention (+ split combine),
    # LM head, accept (records from the head's keys + accept), compaction (2), page release, next roots
    launches_per_step = 10 + (1 if attn_ws.numel() > 256 else 0)
    logits = torch.empty(B * MAX_NODES, VOCAB, dtype=torch.bfloat16, device=dev)
    keys = torch.empty(B * MAX_NODES, (VOCAB + 2047) // 2048, dtype=torch.int64, device=dev)
    lmh_ws = a11spec.ops.workspace(256, dev)
    uni = torch.empty(B, MAX_NODES, dtype=torch.float32, device=dev)
    acc = a11spec.ops.alloc_accept(a11spec.STOCH_ONEHOT, B, MAX_NODES, VOCAB, dev)
    freed = torch.full_like(page_table, -1)
    n_freed = torch.zeros(B, dtype=torch.int32, device=dev)
    kv_ws = a11spec.ops.workspace(256, dev)
    grown = torch.empty(B, dtype=torch.int32, device=dev)
    ev_kernels = []  # per timed step: (attention start, end, accept start, end)

    # Acceptance counters: K3 accumulates them on the device every step; every
    # REDUCE_EVERY steps a snapshot is all-reduced over the ranks on a side
    # stream, overlapping the next steps' kernels (a11spec.distributed.CounterReducer).
    from a11spec.distributed import CounterReducer
    reducer = CounterReducer(stats, every=REDUCE_EVERY)

    def step(timed_events=None, inputs=None, ready=None, out_free=None):
        # inputs: (hidden, q, last, uniforms) of this step; default the resident
        # set with uniforms drawn on the device. ready: events of the copies of
        # (last, q, hidden, uniforms); each input is waited for just before its
        # first use, so a step starts while its later inputs are still copying.
        # out_free: event after which the acceptance outputs may be rewritten
        # (the previous step's device-to-host copy of them has completed).
        hid, qq, lst, un = (hidden, q, last, None) if inputs is None else inputs

        def wait(j):
            if ready is not None:
                torch.cuda.current_stream().wait_event(ready[j])

        wait(0)
        tk, pa, de, nn = a11spec.ngram_expand(table, lst, WIDTH_ROOT, WIDTH_INNER, MAX_DEPTH, MAX_NODES, out=tree)
        grown.copy_(ctx_lens)
        pages.reserve(page_table, grown, nn)  # pages for the tree slots ctx_lens + i
        evs = None
        if timed_events is not None:
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            evs[0].record()
        wait(1)
        a11spec.tree_attention(qq, k_pool, v_pool, page_table, ctx_lens, pa, nn, max_kv_len=max_kv,
                               out=attn_out, ws=attn_ws)
        if evs:
            evs[1].record()
        wait(2)
        if evs:
            evs[4].record()
        # K7: logits and the acceptance's chunk keys in one tcgen05 GEMM
        a11spec.lm_head(hid, w_out, out=logits, keys=keys, ws=lmh_ws)
        if evs:
            evs[5].record()
        wait(3)
        if un is None:
            uni.uniform_(generator=gen)
            un = uni
        if out_free is not None:
            torch.cuda.current_stream().wait_event(out_free)
        if evs:
            evs[2].record()
        a11spec.accept(a11spec.STOCH_ONEHOT, logits.view(B, MAX_NODES, VOCAB), tk, pa, nn,
                       temperature=TEMP, uniforms=un, stats=stats, out=acc, keys=keys)
        if evs:
            evs[3].record()
            timed_events.append(evs)
        a11spec.kv_compact(k_pool, v_pool, page_table, ctx_lens, acc.accept_len, acc.accepted_nodes,
                           nn, freed_pages=freed, n_freed=n_freed, ws=kv_ws)
        pages.release(freed, n_freed)
        # next root pair: (last accepted token or old root, bonus)
        a11spec.next_roots(tk, acc.accepted_tokens, acc.accept_len, acc.bonus, lst)
        reducer.step()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    s0 = stats.clone()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id(dev)) as clk:
        barrier()
        e_start.record()
        for _ in range(args.steps):
            step(ev_kernels)
        e_end.record()
        barrier()
    ms = e_start.elapsed_time(e_end)
    emitted = int((stats - s0)[STAT_NAMES.index("emitted_tokens")])
    attn_ms = sum(e[0].elapsed_time(e[1]) for e in ev_kernels) / len(ev_kernels)
    acc_ms = sum(e[2].elapsed_time(e[3]) for e in ev_kernels) / len(ev_kernels)
    lmh_ms = sum(e[4].elapsed_time(e[5]) for e in ev_kernels) / len(ev_kernels)

    # end to end through the public API with host buffers: pinned H2D of the
    # step's inputs (hidden states, queries, uniforms, last tokens) and D2H of
    # its results (accepted tokens, lengths, bonus)
    h_hidden = hidden.cpu().pin_memory()
    h_q = q.cpu().pin_memory()
    h_uni = torch.rand(B, MAX_NODES).pin_memory()
    h_last = last.cpu().pin_memory()
    h_out_tok = torch.empty(B, MAX_NODES, dtype=torch.int32).pin_memory()
    h_out_len = torch.empty(B, dtype=torch.int32).pin_memory()
    h_out_bonus = torch.empty(B, dtype=torch.int32).pin_memory()
    bi = sum(t.numel() * t.element_size() for t in (h_hidden, h_q, h_uni, h_last))
    bo = sum(t.numel() * t.element_size() for t in (h_out_tok, h_out_len, h_out_bonus))

    # Two input sets: step k+1's H2D runs on a copy stream while step k
    # computes (a serving loop's double buffering); step k waits for each of
    # its inputs just before the first kernel that reads it, and a set is
    # refilled only after the step that read it.
    copy_stream = torch.cuda.Stream(device=dev)
    ins = [(hidden, q, last, torch.empty_like(uni)),
           (hidden.clone(), q.clone(), last.clone(), torch.empty_like(uni))]
    ready = [[torch.cuda.Event() for _ in range(4)] for _ in range(2)]  # per set: last, q, hidden, uniforms
    free = [torch.cuda.Event(), torch.cuda.Event()]

    def h2d(k):
        hid_d, q_d, last_d, uni_d = ins[k % 2]
        with torch.cuda.stream(copy_stream):
            if k >= 2:
                copy_stream.wait_event(free[k % 2])
            # in order of first use, each with its own event
            for j, (d_, h_) in enumerate(((last_d, h_last), (q_d, h_q), (hid_d, h_hidden), (uni_d, h_uni))):
                d_.copy_(h_, non_blocking=True)
                ready[k % 2][j].record(copy_stream)

    # The results go to the host on a stream of their own, so the next step's
    # kernels do not queue behind the copies; its acceptance waits for them.
    d2h_stream = torch.cuda.Stream(device=dev)
    step_done, out_free = torch.cuda.Event(), torch.cuda.Event()

    def e2e_run(n):
        copy_stream.wait_stream(torch.cuda.current_stream())  # copies start after the timing event
        h2d(0)
        for k in range(n):
            if k + 1 < n:
                h2d(k + 1)
            step(inputs=ins[k % 2], ready=ready[k % 2], out_free=out_free if k > 0 else None)
            free[k % 2].record()
            step_done.record()
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(step_done)
                h_out_tok.copy_(acc.accepted_tokens, non_blocking=True)
                h_out_len.copy_(acc.accept_len, non_blocking=True)
                h_out_bonus.copy_(acc.bonus, non_blocking=True)
                out_free.record(d2h_stream)
        torch.cuda.current_stream().wait_stream(d2h_stream)  # the last results are inside the timed region

    e2e_run(max(1, args.warmup // 2))
    barrier()
    s1 = stats.clone()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id(dev)) as clk_e2e:  # the clock record covers both timed regions
        barrier()
        x0.record()
        e2e_run(args.steps)
        x1.record()
        barrier()
    clk.lines.extend(clk_e2e.lines)
    e2e_ms = x0.elapsed_time(x1)
    e2e_emitted = int((stats - s1)[STAT_NAMES.index("emitted_tokens")])

    reducer.finish()
    torch.cuda.synchronize()
    t = torch.tensor([ms, e2e_ms, attn_ms, acc_ms, lmh_ms], dtype=torch.float64, device=dev)
    cnt = torch.tensor([emitted, e2e_emitted], dtype=torch.int64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(cnt, op=torch.distributed.ReduceOp.SUM)
    ms, e2e_ms, attn_ms, acc_ms, lmh_ms = (float(x) for x in t.tolist())
    emitted, e2e_emitted = (int(x) for x in cnt.tolist())
    if rank != 0:
        return None
    pk = peaks()
    attn_flops = 4.0 * B * HQ * MAX_NODES * (CTX + MAX_NODES / 2) * D  # per launch, tree half-masked
    attn_tflops = attn_flops / (attn_ms * 1e-3) / 1e12
    lmh_flops = 2.0 * B * MAX_NODES * HIDDEN * VOCAB
    lmh_tflops = lmh_flops / (lmh_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": emitted / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; no dataset exists for this path)",
        "config": workload_config(world),
        "mean_emitted_per_seq": emitted / (args.steps * B * world),
        "kernel_us": {"tree_attention": attn_ms * 1e3, "lm_head": lmh_ms * 1e3, "accept": acc_ms * 1e3},
        # the timed region is tens of milliseconds, so the burst GEMM peak is the denominator
        "roofline": {"kernel": "tree_attention", "bound": "tensor", "achieved": attn_tflops,
                     "peak": pk["tflops"], "unit": "TFLOP/s", "frac": attn_tflops / pk["tflops"],
                     "peak_source": f"{pk['src']} bf16 burst", "frac_of_sustained": attn_tflops / pk["tflops_sus"],
                     "traffic": profile_traffic("tree_attention_c5"), "flops_per_launch": attn_flops},
        "roofline_lm_head": {"kernel": "lm_head (chunk keys in the epilogue)", "bound": "tensor",
                             "achieved": lmh_tflops, "peak": pk["tflops"], "unit": "TFLOP/s",
                             "frac": lmh_tflops / pk["tflops"], "peak_source": f"{pk['src']} bf16 burst",
                             "flops_per_launch": lmh_flops,
                             "traffic_small_case": profile_traffic("lm_head_small"),
                             "traffic_case": "2048 x 2048 x 32768 (weight larger than L2), profiles/lm_head_c5.md"},
        "e2e": {"value": e2e_emitted / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": bi,
                "d2h_bytes_per_step": bo},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clk.summary(),
    }
    if reducer.result() is not None:
        line["acceptance_stats_global"] = reducer.result()
    if world == 1 and not args.no_configs:
        cfg = measure_configs(dev, pk, dict(hidden=hidden, w_out=w_out, logits=logits, keys=keys,
                                            tree=(tree[0], tree[1], tree[3], uni)))
        line["configs"] = cfg
        st_ = cfg["C5_accept_stream"]
        line["roofline_accept"] = {"kernel": "accept over the logits (one-hot sampling, T=0.7)", "bound": "hbm",
                                   "achieved": st_["achieved_gbs"], "peak": pk["hbm"], "unit": "GB/s",
                                   "frac": st_["frac_hbm"], "peak_source": f"{pk['src']} HBM copy",
                                   "bytes_per_launch": st_["bytes_per_launch"],
                                   "us_includes": "record init + accept kernel",
                                   "on_step_path": False}
    if host_copy is not None:
        line["cpu_baseline"] = cpu_baseline(host_copy)
    return line


# ----------------------------------------------------------------------------- host path
def host_state(st):
    return {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in st.items()}


class HostStep:
    """The per-GPU C5 step on the host cores, the reference's way where it has
    one:
    * draft trees: the oracle's restatement of the hashed trigram expansion (the
      reference's draft is a formula over the last two tokens,
      engine/speculative.py:13-24, with no table);
    * attention: the decode-attention statements of engine/pipeline.py:391-402
      (query head h reads KV head h // (Hq/Hkv) as repeat_interleave groups them,
      fp32 scores scaled by 1/sqrt(d), softmax, probabilities cast to bf16, PV),
      with the ancestor mask over the tree slots;
    * LM head: hidden x W in fp32 (engine/pipeline.py:471);
    * acceptance: p = softmax(logits / T) (engine/sampler.py:16, 37) of each
      sequence's first-child chain, judged with deterministic drafts (q = 1) by the
      reference's own verifier (src/engine/speculative_verifier.cpp:84-135,
      compiled into oracle/_ref) with its thread_local mt19937(42) uniforms; the
      oracle's restatement of that rule when oracle/_ref is absent. The bonus is
      drawn from the last accepted node's row by torch.multinomial
      (engine/sampler.py:37-38);
    * the accepted K/V rows move to the contiguous slots after the context, which
      grows by the committed tokens, and the next root pair is taken.
    """

    def __init__(self, st):
        import oracle
        self.oracle = oracle
        self.ref = oracle.ref()
        self.table = st["table"].numpy()
        self.log2_buckets = st["log2_buckets"]
        self.last = st["last_tokens"].numpy().copy()
        self.k_pool, self.v_pool = st["k_pool"], st["v_pool"]
        self.q = st["q"]
        self.hidden = st["hidden"]
        self.w32 = st["w"].float()
        pt = st["page_table"].clone()
        # the spare logical pages get the pool's unowned pages, in order
        owned = pt[pt >= 0]
        free = torch.ones(self.k_pool.shape[0], dtype=torch.bool)
        free[owned.long()] = False
        spare = torch.nonzero(free).flatten().int()
        holes = pt < 0
        pt[holes] = spare[: int(holes.sum())]
        self.page_table = pt
        self.ctx = st["ctx_lens"].numpy().astype(np.int64).copy()
        self.gen = torch.Generator().manual_seed(77)
        self.scale = 1.0 / math.sqrt(D)

    @property
    def kind(self) -> str:
        return "reference" if self.ref is not None else "port"

    def _attention(self, b, n, parents):
        L = int(self.ctx[b])
        pos = torch.arange(L + n)
        pages = self.page_table[b, pos // 16].long()
        k = self.k_pool[pages, pos % 16].float()  # [S, Hkv, D]
        v = self.v_pool[pages, pos % 16].float()
        q = self.q[b, :n].float()  # [n, Hq, D]
        allowed = torch.zeros(n, L + n, dtype=torch.bool)
        allowed[:, :L] = True
        for i in range(n):
            a = i
            while a >= 0:
                allowed[i, L + a] = True
                a = int(parents[a]) if a > 0 else -1
        rep = HQ // HKV
        out = torch.empty(n, HQ, D)
        for h in range(HKV):
            qh = q[:, h * rep:(h + 1) * rep].reshape(n * rep, D)
            s = (qh @ k[:, h].T).mul_(self.scale).view(n, rep, L + n)
            s.masked_fill_(~allowed[:, None, :], float("-inf"))
            p = torch.softmax(s, dim=-1).to(torch.bfloat16).float().view(n * rep, L + n)
            out[:, h * rep:(h + 1) * rep] = (p @ v[:, h]).view(n, rep, D)
        return out.to(torch.bfloat16)

    def step(self, seqs) -> int:
        """One step for the sequences `seqs`; returns their emitted tokens."""
        o = self.oracle
        seqs = list(seqs)
        tr = o.ngram_expand(self.table, self.log2_buckets, self.last[seqs], WIDTH_ROOT, WIDTH_INNER,
                            MAX_DEPTH, MAX_NODES)
        rows, chains = [], []
        for s, b in enumerate(seqs):
            n = int(tr["n_nodes"][s])
            par = tr["parents"][s]
            self._attention(b, n, par)
            rows.append(torch.arange(b * MAX_NODES, b * MAX_NODES + n))
            chain = [0]  # the first-child chain from the root
            while True:
                kids = [c for c in range(chain[-1] + 1, n) if par[c] == chain[-1]]
                if not kids:
                    break
                chain.append(kids[0])
            chains.append(chain)
        logits = self.hidden[torch.cat(rows)].float() @ self.w32  # [sum n, V]
        offs = np.concatenate([[0], np.cumsum([len(r) for r in rows])])
        K = max(1, max(len(c) - 1 for c in chains))
        tok = np.zeros((len(seqs), K), np.int32)
        drf = np.ones((len(seqs), K), np.float32)
        tgt = np.zeros((len(seqs), K), np.float32)  # padding is rejected (p = 0)
        for s, chain in enumerate(chains):
            for i in range(1, len(chain)):
                row = logits[offs[s] + chain[i - 1]]
                x = int(tr["tokens"][s, chain[i]])
                tok[s, i - 1] = x
                tgt[s, i - 1] = float(torch.softmax(row / TEMP, dim=-1)[x])
        if self.ref is not None:
            alen = np.zeros(len(seqs), np.uint32)
            self.ref.ref_verify_batch(len(seqs), K, tok, drf, tgt, alen, max(1, torch.get_num_threads()))
            alen = alen.astype(np.int64)
        else:
            alen = o.verify_chain(drf, tgt, np.random.default_rng(42).random(tgt.shape, dtype=np.float32))[0]
        emitted = 0
        for s, b in enumerate(seqs):
            chain, a = chains[s], int(min(alen[s], len(chains[s]) - 1))
            probs = torch.softmax(logits[offs[s] + chain[a]] / TEMP, dim=-1)
            bonus = int(torch.multinomial(probs, 1, generator=self.gen))
            L = int(self.ctx[b])
            for j in range(a):  # accepted node chain[j+1] moves from slot L + node to L + 1 + j
                src, dst = L + chain[j + 1], L + 1 + j
                ps, pd = self.page_table[b, src // 16].long(), self.page_table[b, dst // 16].long()
                self.k_pool[pd, dst % 16] = self.k_pool[ps, src % 16]
                self.v_pool[pd, dst % 16] = self.v_pool[ps, src % 16]
            self.ctx[b] = L + 1 + a
            newest = int(tr["tokens"][s, chain[a]])  # last accepted token, or the old root
            self.last[b] = (newest, bonus)
            emitted += a + 1
        return emitted


def cpu_baseline(hs) -> dict:
    """The host path on a bounded sample of the per-GPU step (rank 0, one GPU)."""
    path = HostStep(hs)
    threads = torch.get_num_threads()
    path.step([B_PER_GPU - 1])  # warm-up (thread pools, first-touch pages)
    sample = list(range(8))
    t0 = time.perf_counter()
    emitted = path.step(sample)
    dt = time.perf_counter() - t0
    return {"value": emitted / dt, "unit": UNIT, "cores": threads, "kind": path.kind,
            "sample": f"{len(sample)} of the {B_PER_GPU} sequences of one per-GPU step after a one-sequence "
                      f"warm-up, {dt:.1f} s: trigram expansion (oracle), tree attention over ctx {CTX} and the "
                      f"LM head in torch on {threads} threads, acceptance by the "
                      f"{'reference verifier' if path.kind == 'reference' else 'oracle restatement'}"}


HOST_SAMPLE = 8  # sequences of the per-GPU step that one host step processes


def run_reference(args, rank, world):
    """The per-GPU step on the host cores (HostStep), on the arm's metric and
    config. Each step is a bounded sample: HOST_SAMPLE of the 32 sequences,
    rotating so that consecutive steps cover all of them; a sequence's host cost
    does not depend on which others share its step, so tokens/s is the rate of
    the whole step."""
    if rank != 0:
        return None
    W = workloads_module()
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    st = host_state(W.make_c5(seed=5, batch=B_PER_GPU, ctx=CTX, device="cpu", spare_pages=SPARE_PAGES))
    path = HostStep(st)

    def seqs(k):
        return [(k * HOST_SAMPLE + i) % B_PER_GPU for i in range(HOST_SAMPLE)]

    for k in range(args.warmup):
        path.step(seqs(k))
    t0 = time.perf_counter()
    emitted = 0
    for k in range(args.steps):
        emitted += path.step(seqs(args.warmup + k))
    dt = time.perf_counter() - t0
    v = emitted / dt
    return {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic (seeded; no dataset exists for this path)",
            "config": workload_config(world),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": path.kind,
                             "sample": f"each step {HOST_SAMPLE} of the {B_PER_GPU} sequences of the per-GPU "
                                       f"step, rotating over all of them; trigram expansion (oracle), attention, "
                                       f"LM head and sampler in torch fp32, acceptance by the "
                                       f"{'reference verifier' if path.kind == 'reference' else 'oracle'}"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true")
    args = ap.parse_args()
    # The JSON line is the only thing on stdout: file descriptor 1 points at
    # stderr for the run (libraries such as NCCL print banners there) and the
    # line goes to a saved copy of the real stdout.
    sys.stdout.flush()
    result_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    line = run_reference(args, rank, world) if args.impl == "reference" else run_ours(args, rank, world, local_rank)
    if line is not None:
        print(json.dumps(line), file=result_out, flush=True)
    if world > 1 and args.impl == "ours":
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
