"""Benchmark of the speculative-decoding hot path (one JSON line on rank 0).

Workload (per GPU, weak scaling): the end-to-end draft -> verify -> accept
step of 32 sequences: hashed trigram drafting (2^20 x 8 table, Zipf(1.2)
counts) into trees of <= 64 nodes (4 at depth 1, 2 below, depth <= 5), tree
attention over 16-token KV pages with context 32768 (GQA 32/4, d=128, bf16),
the LM head [nodes, 2048] x [2048, 151936] (bf16, torch/cuBLAS input stage),
sampling acceptance at T=0.7 with seeded uniforms, and KV compaction. Inputs are
seeded synthetic tensors (no dataset exists for this path).

metric: accepted tokens/s (emitted tokens = accepted drafts + bonus, summed over
all ranks, over the max-over-ranks device time).

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Multi-GPU: launched by torch.distributed.run, one rank per GPU, NCCL only for
the per-step acceptance counters.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "a11-llm-optimizer_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "accepted tokens/s"
UNIT = "tokens/s"
B_PER_GPU, CTX, MAX_NODES, HQ, HKV, D, HIDDEN, VOCAB, TEMP = 32, 32768, 64, 32, 4, 128, 2048, 151936, 0.7
WIDTH_ROOT, WIDTH_INNER, MAX_DEPTH = 4, 2, 5
SPARE_PAGES = 32  # per sequence: room for the context to grow by the committed tokens
LOG2_BUCKETS = 20


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
    table, q, hidden, w = st["table"], st["q"], st["hidden"], st["w"]
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
    # accept (record init + accept), compaction (2), page release, next roots
    launches_per_step = 9 + (1 if attn_ws.numel() > 256 else 0)
    logits = torch.empty(B * MAX_NODES, VOCAB, dtype=torch.bfloat16, device=dev)
    uni = torch.empty(B, MAX_NODES, dtype=torch.float32, device=dev)
    acc = a11spec.ops.alloc_accept(a11spec.STOCH_ONEHOT, B, MAX_NODES, VOCAB, dev)
    freed = torch.full_like(page_table, -1)
    n_freed = torch.zeros(B, dtype=torch.int32, device=dev)
    kv_ws = a11spec.ops.workspace(256, dev)
    grown = torch.empty(B, dtype=torch.int32, device=dev)
    ev_attn = []

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
        if timed_events is not None:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        wait(1)
        a11spec.tree_attention(qq, k_pool, v_pool, page_table, ctx_lens, pa, nn, max_kv_len=max_kv,
                               out=attn_out, ws=attn_ws)
        if timed_events is not None:
            e1.record()
            timed_events.append((e0, e1))
        wait(2)
        torch.matmul(hid, w, out=logits)
        wait(3)
        if un is None:
            uni.uniform_(generator=gen)
            un = uni
        if out_free is not None:
            torch.cuda.current_stream().wait_event(out_free)
        a11spec.accept(a11spec.STOCH_ONEHOT, logits.view(B, MAX_NODES, VOCAB), tk, pa, nn,
                       temperature=TEMP, uniforms=un, stats=stats, out=acc)
        a11spec.kv_compact(k_pool, v_pool, page_table, ctx_lens, acc.accept_len, acc.accepted_nodes,
                           nn, freed_pages=freed, n_freed=n_freed, ws=kv_ws)
        pages.release(freed, n_freed)
        # next root pair: (last accepted token or old root, bonus)
        a11spec.next_roots(tk, acc.accepted_tokens, acc.accept_len, acc.bonus, lst)
        if world > 1:
            torch.distributed.all_reduce(stats.clone(), op=torch.distributed.ReduceOp.SUM)

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
            step(ev_attn)
        e_end.record()
        barrier()
    ms = e_start.elapsed_time(e_end)
    emitted = int((stats - s0)[a11spec.STAT_NAMES.index("emitted_tokens")])
    attn_ms = sum(a.elapsed_time(b) for a, b in ev_attn) / len(ev_attn)

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
    e2e_emitted = int((stats - s1)[a11spec.STAT_NAMES.index("emitted_tokens")])

    t = torch.tensor([ms, e2e_ms, attn_ms], dtype=torch.float64, device=dev)
    cnt = torch.tensor([emitted, e2e_emitted], dtype=torch.int64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(cnt, op=torch.distributed.ReduceOp.SUM)
    ms, e2e_ms, attn_ms = (float(x) for x in t.tolist())
    emitted, e2e_emitted = (int(x) for x in cnt.tolist())
    if rank != 0:
        return None
    pk = peaks()
    attn_flops = 4.0 * B * HQ * MAX_NODES * (CTX + MAX_NODES / 2) * D  # per launch, tree half-masked
    attn_tflops = attn_flops / (attn_ms * 1e-3) / 1e12
    traffic = profile_traffic("tree_attention_c5")
    line = {
        "metric": METRIC, "value": emitted / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; no dataset exists for this path)",
        "config": {"workload": "C5 end-to-end draft->reserve pages->verify->accept->compact->release pages, "
                               "32 seqs/GPU, context growing from 32768 by the committed tokens",
                   "seqs_per_gpu": B, "global_seqs": B * world, "ctx": CTX, "max_nodes": MAX_NODES,
                   "gqa": f"{HQ}/{HKV}", "head_dim": D, "vocab": VOCAB, "temperature": TEMP,
                   "parallelism": f"request-batch dp{world}",
                   "l2": "inputs larger than L2 (2.15 GB KV + 622 MB logits per step)"},
        "mean_emitted_per_seq": emitted / (args.steps * B * world),
        "kernel_us": {"tree_attention": attn_ms * 1e3},
        "roofline": {"kernel": "tree_attention", "bound": "tensor", "achieved": attn_tflops,
                     "peak": pk["tflops_sus"], "unit": "TFLOP/s", "frac": attn_tflops / pk["tflops_sus"],
                     "peak_source": f"{pk['src']} bf16 sustained", "traffic": traffic,
                     "flops_per_launch": attn_flops},
        "e2e": {"value": e2e_emitted / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": bi,
                "d2h_bytes_per_step": bo},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(st, args)
    return line


# ----------------------------------------------------------------------------- CPU paths
def cpu_path_one_sequence(st, b, use_ref_verifier):
    """The whole path for sequence b on the host: trigram expansion (oracle),
    tree attention in torch exactly as engine/pipeline.py:391-402 computes it,
    LM head, softmax, acceptance (reference verifier on the chain decisions
    where it is built, else the oracle), compaction (oracle). Returns emitted
    tokens."""
    import oracle
    table = st["table_np"]
    last = st["last_np"][b:b + 1]
    tr = oracle.ngram_expand(table, st["log2_buckets"], last, WIDTH_ROOT, WIDTH_INNER, MAX_DEPTH, MAX_NODES)
    n = int(tr["n_nodes"][0])
    par = tr["parents"][0]
    # attention: gather this sequence's KV (fp32) and compute per node
    pt = st["page_table_np"][b]
    L = CTX
    pos = np.arange(L + n)
    pages = torch.from_numpy(pt[pos // 16].astype(np.int64))
    slots = torch.from_numpy(pos % 16)
    kk = st["k_pool"][pages, slots].float()  # [S, Hkv, D]
    vv = st["v_pool"][pages, slots].float()
    rep = HQ // HKV
    kk = kk.repeat_interleave(rep, dim=1)
    vv = vv.repeat_interleave(rep, dim=1)
    q = st["q"][b, :n].float()  # [n, Hq, D]
    scores = torch.einsum("nhd,shd->nhs", q, kk) / np.sqrt(D)
    mask = torch.zeros(n, L + n, dtype=torch.bool)
    for i in range(n):
        a = i
        while a >= 0:
            mask[i, L + a] = True
            a = int(par[a]) if a > 0 else -1
    mask[:, :L] = True
    scores.masked_fill_(~mask[:, None, :], float("-inf"))
    probs = torch.softmax(scores, dim=-1).to(torch.bfloat16).float()
    _ = torch.einsum("nhs,shd->nhd", probs, vv)
    logits = st["hidden"][b * MAX_NODES: b * MAX_NODES + n].float() @ st["w"]
    uni = np.random.default_rng(b).random((1, MAX_NODES), dtype=np.float32)
    tgt = np.zeros((1, MAX_NODES, VOCAB), np.float32)
    tgt[0, :n] = logits.numpy()
    r = oracle.accept(1, tgt, tr["tokens"], tr["parents"], tr["n_nodes"], temperature=TEMP, uniforms=uni)
    if use_ref_verifier and oracle.ref() is not None:
        # the reference verifier judges the first-child chain on the same probabilities
        chain = [1]
        while True:
            kids = [c for c in range(chain[-1] + 1, n) if par[c] == chain[-1]]
            if not kids:
                break
            chain.append(kids[0])
        probs_chain = r["node_probs"][0, chain].astype(np.float32)
        oracle.ref_verify(tr["tokens"][0, chain], np.ones(len(chain), np.float32), probs_chain)
    return int(r["accept_len"][0]) + 1


def host_state(st):
    return dict(table_np=st["table"].cpu().numpy(), log2_buckets=st["log2_buckets"],
                last_np=st["last_tokens"].cpu().numpy(), page_table_np=st["page_table"].cpu().numpy(),
                k_pool=st["k_pool"].cpu(), v_pool=st["v_pool"].cpu(), q=st["q"].cpu(),
                hidden=st["hidden"].cpu(), w=st["w"].cpu().float())


def cpu_baseline(st, args):
    hs = host_state(st)
    threads = torch.get_num_threads()
    t0 = time.perf_counter()
    emitted = cpu_path_one_sequence(hs, 0, use_ref_verifier=False)
    dt = time.perf_counter() - t0
    return {"value": emitted / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"1 of {B_PER_GPU} sequences of the per-GPU workload (whole path: trigram "
                      f"expansion, tree attention over ctx {CTX}, LM head, sampling acceptance), "
                      f"{dt:.1f} s; torch CPU ops for attention/LM head on {threads} threads, C oracle "
                      f"for the rest"}


def run_reference(args, rank, world):
    """CPU path of the reference (its attention math engine/pipeline.py:391-402 in
    torch, its verifier src/engine/speculative_verifier.cpp for the chain decisions)
    with the oracle port for the parts the reference lacks."""
    if rank != 0:
        return None
    import oracle
    from a11spec import workloads as W
    st = W.make_c5(seed=5, batch=B_PER_GPU, ctx=CTX, device="cpu")
    hs = host_state(st)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref_built = oracle.ref() is not None
    for i in range(args.warmup):
        cpu_path_one_sequence(hs, i % B_PER_GPU, ref_built)
    t0 = time.perf_counter()
    emitted = 0
    for i in range(args.steps):
        emitted += cpu_path_one_sequence(hs, i % B_PER_GPU, ref_built)
    dt = time.perf_counter() - t0
    v = emitted / dt
    return {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic (seeded)",
            "config": {"workload": "C5 end-to-end, one sequence per step (bounded sample)",
                       "ctx": CTX, "max_nodes": MAX_NODES, "vocab": VOCAB},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads,
                             "kind": "reference" if ref_built else "port",
                             "sample": "one sequence of the 32-sequence per-GPU workload per step"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
