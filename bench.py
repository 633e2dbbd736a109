"""Committed tokens/s of the speculative draft -> verify -> accept -> commit step.

Default workload (N=1 and per rank at N>1, weak scaling): the GPT-2-small-shaped
pair in bf16 (target d768/12L/12H/ff3072, draft d384/4L/6H/ff1536, vocab
32000, random-init weights, seed 0), 256 concurrent requests with prompts of
U[128,1024] synthetic tokens, k=5, block 16, greedy.  A step is one
``batched_speculative_step`` over the 256 active rows.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl pse|reference]

Rank 0 prints one JSON line.  ``value`` times K steps replayed from the
captured CUDA graph with everything resident in HBM (CUDA events, max over
ranks); ``e2e`` times K further steps through the public Python API
(request ids in, accepted tokens out, one host<->device round trip per step).
``roofline`` is the verify-attention kernel (the step's largest HBM stream)
timed live on the same cache state; ``cpu_baseline`` is the reference's CPU
path (the oracle port, fp32) on a bounded sample.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "paged-speculative-engine_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _tensor_peak():
    """Dense bf16 tensor-core peak in TFLOP/s: the measured burst figure, else
    the fallback measured earlier on this hardware."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index: int, interval_ms: int = 20):
        self.index = index
        self.interval_ms = interval_ms
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.marks: list[float] = []

    def mark(self) -> None:
        """Start / end of a timed region (call in pairs)."""
        self.marks.append(time.perf_counter())

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        windows = list(zip(self.marks[0::2], self.marks[1::2]))
        # a sample reports the interval that ends at its arrival: keep the ones that overlap a timed region
        slack = self.interval_ms / 1000.0
        inside = [ln for t, ln in self.lines if not windows or any(a <= t <= b + slack for a, b in windows)]
        for ln in inside:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "interval_ms": self.interval_ms}


def build_pair(workload, dtype, device, seed=0):
    import pse
    from pse.model import LlamaConfig, ModelConfig, TinyGPT, TinyLlama
    pr = workload.pair
    torch.manual_seed(seed)
    if pr.kind == "gpt":
        d = TinyGPT(ModelConfig(vocab_size=pr.vocab, **pr.draft))
        t = TinyGPT(ModelConfig(vocab_size=pr.vocab, **pr.target))
    else:
        d = TinyLlama(LlamaConfig(vocab_size=pr.vocab, **pr.draft))
        t = TinyLlama(LlamaConfig(vocab_size=pr.vocab, **pr.target))
    return d.eval(), t.eval()


def cache_for(model, workload, n_rows, dtype, device, extra_tokens, prompts=None, n_blocks=None):
    """A pool for n_rows requests of the workload: every row sized for the
    longest prompt, or, given the prompts, for each prompt's own length, or
    ``n_blocks`` blocks."""
    import pse
    cfg = model.cfg
    kv = getattr(cfg, "n_kv_heads", cfg.n_heads)
    hd = cfg.d_model // cfg.n_heads
    bs = workload.block_size
    per_row = workload.prompt_hi + workload.max_new_tokens + extra_tokens
    if prompts is None:
        nb = n_rows * ((per_row + bs - 1) // bs) + 8
    else:
        nb = sum((len(p) + workload.max_new_tokens + extra_tokens + bs - 1) // bs for p in prompts) + 8
    if n_blocks:
        nb = n_blocks
    return pse.PagedKVCache(cfg.n_layers, kv, hd, bs, nb, dtype=dtype, device=device, max_requests=n_rows,
                            max_blocks_per_request=(per_row + bs - 1) // bs)


def run_pse(args, rank, world, device):
    import pse
    import pse._native as N
    from pse import workload as wl
    from pse.speculative import runner_for

    w = wl.WORKLOADS[args.workload]
    dtype = torch.bfloat16 if w.dtype == "bfloat16" else torch.float32
    B = args.rows or w.max_batch_size
    from pse.dist import shard_requests
    from pse.scheduler import Request

    # The job is world x B requests (seeded prompts), sharded LPT-balanced by
    # prompt + max_new tokens: every GPU holds ~B rows (weak scaling).
    allreq = [Request(f"r{i}", p, w.max_new_tokens) for i, p in enumerate(wl.prompts(w, seed=0, n=B * world))]
    mine = shard_requests(allreq, world, rank)
    B = len(mine)
    d, t = build_pair(w, dtype, device)
    if getattr(args, "self_draft", False):
        d = t  # draft == target: every draft accepted at T = 0 (the reference benchmark's ceiling)
    # room for every step the run takes (two structures x (warm-up + K replays + K API steps)), each
    # committing up to k+1 tokens, plus the roofline launch's k+1 reserved tokens
    n_steps = 2 * (max(args.warmup, 3) + 2 * args.steps)
    extra = (w.k + 1) * (n_steps + 1) + w.k + 2
    prompts = [r.prompt_ids for r in mine]
    dc = cache_for(d, w, B, dtype, device, extra, prompts)
    tc = cache_for(t, w, B, dtype, device, extra, prompts)
    rids = [r.request_id for r in mine]
    dn, tn = {}, {}
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = pse.prefill_requests(d, t, dc, tc, rids, prompts)  # batched; same caches as one-by-one calls
    for r in rids:
        dn[r], tn[r] = out[r]
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    prefill_tokens = sum(len(p) for p in prompts)
    k, T = w.k, w.temperature
    # committed tokens of the first rows, over every step of the run (checked against the oracle afterwards)
    n_chk = min(2, B)
    chk_tokens = {r: [] for r in rids[:n_chk]}

    def api_step(reference_structure):
        nonlocal dn, tn
        if reference_structure:
            res = pse.batched_speculative_step(d, t, rids, dc, tc, dn, tn, k, T, defer_bonus=False)
        else:
            # exactly the reference scheduler's call (engine/scheduler.py:102-105)
            res = pse.batched_speculative_step(d, t, rids, dc, tc, dn, tn, k, T)
        dn, tn = res.draft_next_logits, res.target_next_logits  # what the next step takes back
        for r in chk_tokens:
            chk_tokens[r].extend(res.accepted_tokens[r])
        return sum(map(len, res.accepted_tokens.values()))

    runner = runner_for(d, t, dc, tc, k)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def sum_ctx(c, slots):
        return int(c._blocks.seq_len[slots.long()].sum().item())

    def measure(reference_structure):
        """W >= 3 warm-up steps through the API (eager runs, then the CUDA-graph
        capture of the steady-state step; each of that step's kernels is
        counted once, in its eager run), K timed graph replays (inputs
        resident), then K timed steps through the public API.  The default
        structure's first step runs from rows just prefilled (width-k verify,
        bonus deferred); from the second on every row is pending (width-k+1
        verify from the pending position)."""
        api_step(reference_structure)
        before = sum(N.launches.values())
        api_step(reference_structure)
        kernels = sum(N.launches.values()) - before
        for _ in range(max(args.warmup, 3) - 2):
            api_step(reference_structure)
        if args.profile_step:
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push("pse_step")
            pse.batched_speculative_step(d, t, rids, dc, tc, dn, tn, k, T, use_graph=False,
                                         defer_bonus=False if reference_structure else None)
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
            return None
        steady = (False, False) if reference_structure else (True, True)  # (rows pending in, bonus deferred out)
        graph = [g for key, g in runner.graphs.items() if key[0] == B and key[3:5] == steady][0]
        b = runner.bufs[B]
        nacc_hist = torch.zeros(args.steps, B, dtype=torch.int32, device=device)
        tok_hist = torch.zeros(args.steps, n_chk, k + 1, dtype=torch.int32, device=device)
        ctx0 = (sum_ctx(dc, b.slots_d), sum_ctx(tc, b.slots_t))
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk.mark()
        e0.record()
        for s in range(args.steps):
            graph.replay()
            nacc_hist[s].copy_(b.n_acc)
            tok_hist[s].copy_(b.tokens[:n_chk])
        e1.record()
        barrier()
        clk.mark()
        ms = e0.elapsed_time(e1)
        th, nh = tok_hist.cpu().numpy(), nacc_hist[:, :n_chk].cpu().numpy()
        for s in range(args.steps):
            for i, r in enumerate(rids[:n_chk]):
                chk_tokens[r].extend(th[s, i, :nh[s, i] + 1].tolist())
        ctx1 = (sum_ctx(dc, b.slots_d), sum_ctx(tc, b.slots_t))
        committed = int(nacc_hist.sum().item()) + args.steps * B
        # rows of the timed steps by number of drafts accepted (0..k)
        acc_hist = np.bincount(nacc_hist.cpu().numpy().ravel().clip(0, k), minlength=k + 1).tolist()
        for c in (dc, tc):  # host mirrors of the lengths after the replays
            c._resync_lengths()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        e2e_tokens = sum(api_step(reference_structure) for _ in range(args.steps))
        f1.record()
        barrier()
        return dict(ms=ms, committed=committed, e2e_ms=f0.elapsed_time(f1), e2e_tokens=e2e_tokens,
                    kernels=kernels, ctx_mean=((ctx0[0] + ctx1[0]) / 2, (ctx0[1] + ctx1[1]) / 2),
                    acc_hist=acc_hist)

    if args.profile_step:
        return measure(args.reference_structure)
    # clocks are sampled from before the first warm-up to the end of the last timed region;
    # the summary keeps the samples taken inside the timed regions
    with ClockSampler(device.index or 0) as clk:
        ref = measure(True)  # the reference's step structure: 2 target + k+1 draft calls
        head = ref if args.reference_structure else measure(False)  # 1 target call of width k+1 + k+1 draft calls
    head["clocks"] = clk.summary()
    b = runner.bufs[B]
    width = k if args.reference_structure else k + 1

    # ---- verify-attention kernel, timed live on the current target state ----
    dm = runner.dm_t
    hd, hq, hk = dm.head_dim, dm.q_heads, dm.kv_heads
    lens = tc._blocks.seq_len[b.slots_t.long()]
    base = lens.to(torch.int32)
    ctx = (base + width).to(torch.int64)
    max_ctx = int(ctx.max().item())
    q = torch.randn(B * width, hq * hd, dtype=dtype, device=device)
    out = torch.empty_like(q)
    wsb = N.size_call("pse_paged_attention_workspace", B, width, hq, hk, hd, max_ctx)
    ws = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=device)
    st = N.stream_ptr()
    reps = 20
    # the timed launches read blocks up to base + width: reserve them so every page read is a table entry
    N.call("pse_kv_reserve", tc.state, b.slots_t.data_ptr(), B, width, b.base[0].data_ptr(), st)

    # rows handed out longest first, as the step's own attention calls do
    order = torch.argsort(-base.to(torch.int64), stable=True).to(torch.int32)

    def attn_all_layers():
        for li in range(dm.n_layers):
            N.call("pse_paged_attention", tc.state, tc.layer(li), q.data_ptr(), q.stride(0), out.data_ptr(),
                   out.stride(0), b.slots_t.data_ptr(), base.data_ptr(), B, width, hq, 1.0 / math.sqrt(hd),
                   max_ctx, order.data_ptr(), ws.data_ptr(), ws.numel(), st)

    attn_all_layers()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for _ in range(reps):
        attn_all_layers()
    a1.record()
    torch.cuda.synchronize()
    attn_ms = a0.elapsed_time(a1) / (reps * dm.n_layers)
    esize = torch.finfo(dtype).bits // 8
    attn_bytes = int(ctx.sum().item()) * hk * hd * 2 * esize + 2 * q.numel() * esize + B * 4 * tc.max_blocks

    # ---- KV + weight bytes of the minimal step (1 target pass of width k+1, k draft passes) ----
    def kv_bytes_per_token(m):
        c = m.cfg
        return 2 * c.n_layers * getattr(c, "n_kv_heads", c.n_heads) * (c.d_model // c.n_heads) * esize

    w_t = sum(p.numel() for p in t.parameters()) * esize
    w_d = sum(p.numel() for p in d.parameters()) * esize
    step_bytes = (w_t + head["ctx_mean"][1] * kv_bytes_per_token(t)
                  + k * (w_d + head["ctx_mean"][0] * kv_bytes_per_token(d)))

    # host <-> device bytes of one API step, counted from the buffers it copies:
    # the whole per-row input buffer in, the whole packed result out
    sb = runner.bufs[B]
    h2d = sb.host_in.numel() * sb.host_in.element_size()
    d2h = sb.host_pack.numel() * sb.host_pack.element_size()

    from pse.dist import reduce_stats
    out = {}
    for name, m in (("ref", ref), ("head", head)):
        c_, s_, _ = reduce_stats(m["committed"], m["ms"] / 1000.0, device=device)
        e_, es_, _ = reduce_stats(m["e2e_tokens"], m["e2e_ms"] / 1000.0, device=device)
        out[name] = dict(committed=c_, ms=s_ * 1000.0, e2e_tokens=e_, e2e_ms=es_ * 1000.0)
    return dict(ref=out["ref"], head=out["head"], attn_ms=attn_ms, attn_bytes=attn_bytes, attn_width=width,
                prefill_s=prefill_s, prefill_tokens=prefill_tokens, clocks=head["clocks"], B=B, k=k, kernels_per_step=head["kernels"],
                dtype=str(dtype), h2d=h2d, d2h=d2h, step_bytes=step_bytes,
                tokens_per_step_mean=head["committed"] / args.steps / max(world, 1),
                deferred=not args.reference_structure, acc_hist=head["acc_hist"],
                check_rows=[(prompts[i], chk_tokens[rids[i]]) for i in range(n_chk)])


def token_check(args, rows, threads):
    """Greedy parity of committed tokens from the timed run: for each checked
    row, one teacher-forced forward of the oracle (fp32 CPU model on the same
    weights rounded to bf16) over prompt + everything the row committed; each
    committed token must be the oracle's argmax given the same prefix or lie
    within the bf16 logit tolerance of it (the oracle of engine/generate.py:
    24-38 takes the argmax)."""
    from oracle.model import LlamaConfig, ModelConfig, TinyGPT, TinyLlama
    from pse import workload as wl
    w = wl.WORKLOADS[args.workload]
    if w.temperature > 0 or not rows:
        return None
    torch.set_num_threads(threads)
    pr = w.pair
    torch.manual_seed(0)
    if pr.kind == "gpt":
        TinyGPT(ModelConfig(vocab_size=pr.vocab, **pr.draft))  # same RNG stream as the engine's pair
        t = TinyGPT(ModelConfig(vocab_size=pr.vocab, **pr.target)).eval()
    else:
        TinyLlama(LlamaConfig(vocab_size=pr.vocab, **pr.draft))
        t = TinyLlama(LlamaConfig(vocab_size=pr.vocab, **pr.target)).eval()
    with torch.no_grad():
        for p in t.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    n_tok, n_div, worst = 0, 0, 0.0
    for prompt, gen in rows:
        with torch.no_grad():
            ol = t(torch.tensor([list(prompt) + gen[:-1]]))[0][0][len(prompt) - 1:]
        g = torch.tensor(gen)
        gap = ol.max(dim=-1).values - ol.gather(1, g.view(-1, 1)).view(-1)
        n_tok += len(gen)
        n_div += int((ol.argmax(dim=-1) != g).sum())
        worst = max(worst, float(gap.max()))
    return {"rows": len(rows), "tokens": n_tok, "not_oracle_argmax": n_div, "max_logit_gap": worst,
            "tolerance": 2e-2, "ok": worst < 2e-2}


def cpu_reference(args, sample_rows, sample_steps, threads, warmup=0):
    """The reference's CPU path (the oracle port of engine/*.py, fp32) on a
    sample of the same workload: ``sample_steps`` batched speculative steps
    over the workload's first ``sample_rows`` rows after ``warmup`` untimed
    ones.  Rows start at their prompts' lengths.  Where the prompts hold more
    than ``CPU_PREFILL_TOKENS`` tokens in all, the per-request CPU prefill
    (minutes at 256 rows) is replaced by appending seeded N(0,1) K/V of each
    prompt's length and seeded next-token logits: a step's work depends on
    the rows' lengths, not on the cached values, and with random-init models
    the committed tokens per row are ~1 per step either way."""
    from oracle.model import LlamaConfig, ModelConfig, TinyGPT, TinyLlama
    from oracle.paged_cache import PagedKVCache
    from oracle.speculative import batched_speculative_step, prefill_request
    from pse import workload as wl

    torch.set_num_threads(threads)
    w = wl.WORKLOADS[args.workload]
    pr = w.pair
    torch.manual_seed(0)
    if pr.kind == "gpt":
        d = TinyGPT(ModelConfig(vocab_size=pr.vocab, **pr.draft)).eval()
        t = TinyGPT(ModelConfig(vocab_size=pr.vocab, **pr.target)).eval()
    else:
        d = TinyLlama(LlamaConfig(vocab_size=pr.vocab, **pr.draft)).eval()
        t = TinyLlama(LlamaConfig(vocab_size=pr.vocab, **pr.target)).eval()
    prompts = wl.prompts(w, seed=0, n=sample_rows)
    steps_total = warmup + sample_steps

    def mk(m):
        c = m.cfg
        kv = getattr(c, "n_kv_heads", c.n_heads)
        nb = sum((len(p) + (w.k + 1) * (steps_total + 1) + w.block_size - 1) // w.block_size for p in prompts) + 8
        return PagedKVCache(c.n_layers, kv, c.d_model // c.n_heads, w.block_size, nb)

    dc, tc = mk(d), mk(t)
    rids = [f"c{i}" for i in range(sample_rows)]
    dn, tn = {}, {}
    synthetic = sum(len(p) for p in prompts) > CPU_PREFILL_TOKENS
    if not synthetic:
        for r, p in zip(rids, prompts):
            dn[r], tn[r] = prefill_request(d, t, dc, tc, r, p)
    else:
        g = torch.Generator().manual_seed(0)
        longest = max(len(p) for p in prompts)
        for m, c, nxt in ((d, dc, dn), (t, tc, tn)):
            cfg = m.cfg
            kv, hd = getattr(cfg, "n_kv_heads", cfg.n_heads), cfg.d_model // cfg.n_heads
            src_k = torch.randn(cfg.n_layers, kv, longest, hd, generator=g)
            src_v = torch.randn(cfg.n_layers, kv, longest, hd, generator=g)
            for r, p in zip(rids, prompts):
                c.create_request(r)
                n = len(p)
                c.append(r, [src_k[l, :, :n] for l in range(cfg.n_layers)],
                         [src_v[l, :, :n] for l in range(cfg.n_layers)])
                nxt[r] = torch.randn(pr.vocab, generator=g)
    for _ in range(warmup):
        res = batched_speculative_step(d, t, rids, dc, tc, dn, tn, w.k, w.temperature)
        dn, tn = res.draft_next_logits, res.target_next_logits
    tok = 0
    t0 = time.perf_counter()
    for _ in range(sample_steps):
        res = batched_speculative_step(d, t, rids, dc, tc, dn, tn, w.k, w.temperature)
        tok += sum(len(v) for v in res.accepted_tokens.values())
        dn, tn = res.draft_next_logits, res.target_next_logits
    dt = time.perf_counter() - t0
    start = ("rows start from seeded random K/V and next logits of their prompts' lengths (the per-request CPU "
             "prefill is not run)" if synthetic else "prefill untimed")
    return dict(value=tok / dt, tokens=tok, seconds=dt, cores=threads,
                sample=f"{sample_rows} of {w.max_batch_size} rows x {sample_steps} batched steps of the {w.name} "
                       f"workload (its first {sample_rows} prompts, after {warmup} untimed steps), fp32 oracle "
                       f"port of the reference's step, {threads} threads; {start}")


CPU_PREFILL_TOKENS = 16384  # above this many prompt tokens the CPU sample starts from synthetic K/V


# ncu dram__bytes_read.sum + dram__bytes_write.sum over the algorithmic bytes of
# attn_tc_kernel, captured on the gpt2-verify microbench shape (the summary
# with the command is profiles/attn_tc_gpt2-verify.md); keyed by (workload,
# verify width).
ATTN_TRAFFIC_RATIO: dict = {("gpt2-small", 6): (481297920 + 5749760) / 477461504}

ATTN_SHAPES = {
    # name: rows, width, q_heads, kv_heads, head_dim, block, ctx_lo, ctx_hi (ctx includes the width queries)
    "gpt2-verify": (256, 6, 12, 12, 64, 16, 134, 1030),
    "gpt2-verify5": (256, 5, 12, 12, 64, 16, 133, 1029),
    "gpt2-verify-bs64": (256, 6, 12, 12, 64, 64, 134, 1030),
    "llama-verify": (512, 5, 32, 8, 64, 32, 133, 8197),
    "gpt2-draft-bs64": (256, 1, 6, 6, 64, 64, 129, 1025),
    "gpt2-draft": (256, 1, 6, 6, 64, 16, 129, 1025),
    "verify-5a": (1024, 8, 32, 8, 128, 16, 512, 32768),
    # prompt prefill (width = context: each prompt attends to itself, causal)
    "gpt2-prefill": (32, 512, 12, 12, 64, 16, 512, 512),
    "llama-prefill": (8, 2048, 32, 8, 64, 32, 2048, 2048),
    "prefill-hd128": (8, 2048, 32, 8, 128, 16, 2048, 2048),
}


def micro_attention(args, device, emit=True):
    """Verify-attention kernel microbenchmark: one layer's pools, block tables a
    random permutation of a shared pool, Q/K/V ~ N(0,1), bf16.  Bytes are the
    algorithmic K/V bytes (sum of contexts x kv_heads x head_dim x 2 x 2 B) plus
    Q and O; each timed launch reads a pool far larger than L2 (except the small
    row counts of a size sweep).  ``--steps`` launches are captured in one CUDA
    graph and timed as one replay (device time)."""
    import pse
    import pse._native as N
    rows, width, hq, hk, hd, bs, lo, hi = ATTN_SHAPES[args.attn_shape]
    if args.rows:
        rows = args.rows
    rng = np.random.default_rng(0)
    ctx = rng.integers(lo, hi + 1, size=rows)
    need = (ctx + bs - 1) // bs
    nb = int(need.sum())
    c = pse.PagedKVCache(1, hk, hd, bs, nb, dtype=torch.bfloat16, device=device, max_requests=rows,
                         max_blocks_per_request=int(need.max()))
    perm = torch.from_numpy((rng.permutation(nb) if args.attn_pages == "permuted" else np.arange(nb)).astype(np.int32))
    table = torch.full((rows, int(need.max())), -1, dtype=torch.int32)
    o = 0
    for i, n in enumerate(need):
        table[i, :n] = perm[o:o + n]
        o += n
    c._blocks.block_table.copy_(table)
    c._blocks.nblocks.copy_(torch.from_numpy(need.astype(np.int32)))
    g = torch.Generator(device=device).manual_seed(1)
    c.k_pool.normal_(generator=g)
    c.v_pool.normal_(generator=g)
    q = torch.randn(rows * width, hq * hd, device=device, generator=g).to(torch.bfloat16)
    out = torch.empty_like(q)
    slots = torch.arange(rows, dtype=torch.int32, device=device)
    base = torch.from_numpy((ctx - width).astype(np.int32)).to(device)
    max_ctx = int(ctx.max())
    wsb = N.size_call("pse_paged_attention_workspace", rows, width, hq, hk, hd, max_ctx)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=device)
    st = N.stream_ptr()

    # the rows' lengths: everything up to and including the last query
    c._blocks.seq_len.copy_(torch.from_numpy(ctx.astype(np.int32)))
    N.call("pse_attention_prefill_select", {"tc": 0, "off": 1, "single": 2}[args.prefill_kernel])

    def launch():
        N.call("pse_paged_attention", c.state, c.layer(0), q.data_ptr(), q.stride(0), out.data_ptr(), out.stride(0),
               slots.data_ptr(), base.data_ptr(), rows, width, hq, 1.0 / math.sqrt(hd), max_ctx, None, ws.data_ptr(),
               ws.numel(), N.stream_ptr())

    for _ in range(max(args.warmup, 3)):
        launch()
    torch.cuda.synchronize()
    # device time: the launches captured in one CUDA graph (no host dispatch between them)
    graph = torch.cuda.CUDAGraph()
    with N.graph_capture(graph):
        for _ in range(args.steps):
            launch()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clk:
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    kv_bytes = int(ctx.sum()) * hk * hd * 2 * 2
    alg = kv_bytes + 2 * q.numel() * 2 + rows * 4 * int(need.max())
    peak, kind = _peaks()
    gbs = alg / (ms / 1000) / 1e9
    # causal QK^T and PV flops: query w of row i sees base_i + w + 1 keys
    keys = int(sum(int(b) * width + width * (width + 1) // 2 for b in (ctx - width)))
    tflops = 4 * hq * hd * keys / (ms / 1000) / 1e12
    N.call("pse_attention_prefill_select", 0)
    res = {"metric": "paged attention HBM GB/s", "shape": args.attn_shape, "value": gbs, "unit": "GB/s",
                      "frac_of_peak": gbs / peak, "peak": peak, "peak_kind": kind, "us_per_launch": ms * 1000,
                      "tflops": tflops, "tflops_frac_of_bf16_peak": tflops / _tensor_peak()[0],
                      "prefill_kernel": args.prefill_kernel,
                      "algorithmic_bytes": alg, "rows": rows, "width": width, "q_heads": hq, "kv_heads": hk,
                      "head_dim": hd, "block_size": bs, "ctx_mean": float(ctx.mean()), "pages": args.attn_pages,
                      "pool_bytes": 2 * c.k_pool.numel() * 2, "clocks": clk.summary()}
    if emit:
        print(json.dumps(res), flush=True)
    return res


def micro_accept(args, device, emit=True):
    """Accept / resample microbenchmark: fp32 target logits [R, k+1, V] and
    draft logits [R, k, V] ~ N(0, 3^2), V = 128256, R = 1024, k = 8, drafts drawn
    from the draft distributions with explicit uniforms.  Bytes counted are the
    logit rows the rule has to read for the observed outcome: positions 0..n
    of the target and 0..min(n, k-1) of the draft for a row that accepted n
    (at T = 0 only the target rows); the formula figure (2k+1) R V 4 is
    reported beside it."""
    import pse._native as N
    R, k, V, T = args.rows or 1024, 8, 128256, args.temperature
    g = torch.Generator(device=device).manual_seed(0)
    tgt = torch.randn(R, k + 1, V, device=device, generator=g).mul_(3.0)
    drf = torch.randn(k, R, V, device=device, generator=g).mul_(3.0)  # position-major, as the step stores it
    u = torch.rand(R, 2 * k + 1, device=device, dtype=torch.float64, generator=g)
    drafts = torch.empty(R, k, dtype=torch.int32, device=device)
    st = N.stream_ptr()
    for j in range(k):
        N.call("pse_sample_tokens", drf[j].data_ptr(), V, None, R, V, float(T), u.data_ptr(), 2 * k + 1, j,
               drafts.data_ptr() + 4 * j, k, None, 0, st)
    toks = torch.empty(R, k + 1, dtype=torch.int32, device=device)
    nacc = torch.empty(R, dtype=torch.int32, device=device)
    fin = torch.empty(R, dtype=torch.int32, device=device)

    N.load().pse_accept_select(args.accept_kernel)

    def launch():
        N.call("pse_spec_accept", tgt.data_ptr(), (k + 1) * V, None, tgt.data_ptr() + 4 * V, (k + 1) * V, V,
               drf.data_ptr(), V, None, drf.data_ptr() + 4 * R * V, V, R * V, drafts.data_ptr(), u.data_ptr(),
               2 * k + 1, R, k, V, float(T), toks.data_ptr(), nacc.data_ptr(), fin.data_ptr(), st)

    for _ in range(max(args.warmup, 3)):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    n = nacc.long()
    rows_read = (n + 1).sum().item() + (0 if T <= 0 else torch.minimum(n + 1, torch.tensor(k, device=device)).sum().item())
    need = rows_read * V * 4
    formula = (2 * k + 1) * R * V * 4
    peak, kind = _peaks()
    res = {"metric": "accept/resample HBM GB/s", "value": need / (ms / 1000) / 1e9, "unit": "GB/s",
                      "frac_of_peak": need / (ms / 1000) / 1e9 / peak, "peak": peak, "peak_kind": kind,
                      "us_per_launch": ms * 1000, "bytes_needed": need, "bytes_formula_2k+1": formula,
                      "formula_GBps": formula / (ms / 1000) / 1e9, "rows": R, "k": k, "vocab": V, "temperature": T,
                      "mean_accepted": n.float().mean().item(),
                      "kernel": ["cluster-split streaming", "CTA per row (scalar)", "cluster per row (on chip)",
                                 "streaming CTA per row"][args.accept_kernel]
                      if T > 0 else "CTA per row (argmax)"}
    N.load().pse_accept_select(0)
    if emit:
        print(json.dumps(res), flush=True)
    return res


def micro_prefill(args, device):
    """Batched prefill (prefill_requests) against one-by-one prefill_request
    calls on the workload's first ``--rows`` requests (default 64), each into
    fresh caches: wall time with device sync, prompt tokens/s, and whether the
    two left identical block tables and free lists."""
    import pse
    from pse import workload as wl
    w = wl.WORKLOADS[args.workload]
    dtype = torch.bfloat16 if w.dtype == "bfloat16" else torch.float32
    n = args.rows or 64
    prompts = wl.prompts(w, seed=0, n=n)
    ids = [f"r{i}" for i in range(n)]
    d, t = build_pair(w, dtype, device)
    res = {}
    for mode in ("one_by_one", "batched", "batched_again"):
        dc = cache_for(d, w, n, dtype, device, w.k + 2)
        tc = cache_for(t, w, n, dtype, device, w.k + 2)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        if mode == "one_by_one":
            for r, p in zip(ids, prompts):
                pse.prefill_request(d, t, dc, tc, r, p)
        else:
            if mode == "batched_again":
                torch.cuda.nvtx.range_push("prefill_batched")
            pse.prefill_requests(d, t, dc, tc, ids, prompts)
            if mode == "batched_again":
                torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        res[mode] = (time.perf_counter() - t0, [dc.block_table(r) for r in ids] + [tc.block_table(r) for r in ids],
                     dc.allocator.free_list(), tc.allocator.free_list())
        del dc, tc
    tokens = sum(len(p) for p in prompts)
    same = res["one_by_one"][1:] == res["batched"][1:]
    print(json.dumps({"metric": "prefill prompt tokens/s", "workload": w.name, "requests": n, "prompt_tokens": tokens,
                      "one_by_one_s": res["one_by_one"][0], "batched_s": res["batched_again"][0],
                      "one_by_one_tokens_per_s": tokens / res["one_by_one"][0],
                      "batched_tokens_per_s": tokens / res["batched_again"][0],
                      "speedup": res["one_by_one"][0] / res["batched_again"][0],
                      "identical_tables_and_free_lists": same}), flush=True)


def micro_scheduler(args, device, emit=True, warm=True):
    """The whole workload through run_continuous_speculative_batches (FIFO
    admission up to the batch size, batched prefill, steps until every request
    has max_new_tokens, as the reference's own benchmark drives it): committed
    tokens / wall time, device-synchronised, after one untimed run of the same
    workload (graph capture, allocation).  T > 0 draws its uniforms from the
    device Philox stream."""
    import pse
    from pse import workload as wl
    from pse.scheduler import Request
    from pse.dist import reduce_stats, shard_requests
    w = wl.WORKLOADS[args.workload]
    dtype = torch.bfloat16 if w.dtype == "bfloat16" else torch.float32
    world = torch.distributed.get_world_size() if torch.distributed.is_initialized() else 1
    rank = torch.distributed.get_rank() if world > 1 else 0
    n_all = args.rows or w.n_requests
    # the job is n_all requests; with several ranks each runs its LPT shard (strong scaling)
    shard = shard_requests([Request(f"r{i}", p, w.max_new_tokens)
                            for i, p in enumerate(wl.prompts(w, seed=0, n=n_all))], world, rank)
    prompts = [r.prompt_ids for r in shard]
    n = len(prompts)
    batch = args.max_batch or w.max_batch_size
    d, t = build_pair(w, dtype, device)
    if args.sched_mode == "self":
        d = t  # draft == target: every draft accepted (the reference benchmark's ceiling configuration)
    pool_blocks = None
    if args.pool_gb:
        # both pools get the block count that puts pool_gb of the target's K/V on the device
        cfg = t.cfg
        blk = (cfg.n_layers * getattr(cfg, "n_kv_heads", cfg.n_heads) * (cfg.d_model // cfg.n_heads) * 2
               * w.block_size * (2 if dtype == torch.bfloat16 else 4))
        pool_blocks = int(args.pool_gb * 1e9) // blk
    out = {}
    for run in (("warm", "timed") if warm else ("timed",)):
        reqs = [Request(f"{run}{i}", p, w.max_new_tokens) for i, p in enumerate(prompts)]
        dc = cache_for(d, w, n, dtype, device, w.k + 2, prompts, n_blocks=pool_blocks)
        tc = cache_for(t, w, n, dtype, device, w.k + 2, prompts, n_blocks=pool_blocks)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if args.sched_mode == "plain":
            res = pse.run_plain_continuous_batches(t, reqs, tc, batch)
        else:
            res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, batch, k=w.k,
                                                         temperature=w.temperature,
                                                         defer_bonus=False if args.reference_structure else None,
                                                         device_bookkeeping=not args.sched_host_loop)
        e1.record()
        torch.cuda.synchronize()
        # device time from the first launch to the last (the host loop's gaps included)
        out[run] = (e0.elapsed_time(e1) / 1000.0, sum(len(r.output_ids) - len(p) for r, p in
                                                       zip(sorted(res, key=lambda r: int(r.request_id[len(run):])),
                                                           prompts)))
        # the caches hold their step runners (and those their graphs): free
        # the warm-up run's pools before the timed run allocates its own
        del dc, tc, res
        gc.collect()
        torch.cuda.empty_cache()
    secs, toks = out["timed"]
    per_rank = None
    if world > 1:
        toks, secs, per = reduce_stats(toks, secs, None, device=device)
        per_rank = [{"tokens": p[0], "seconds": round(p[1], 3)} for p in per]
    cpu = None
    if not args.no_cpu_baseline and args.sched_mode == "spec" and world == 1:
        # the reference's CPU path (oracle port, fp32) on the same whole workload, all host threads
        from oracle import scheduler as OS
        from oracle.model import ModelConfig as OMC, TinyGPT as OTG, LlamaConfig as OLC, TinyLlama as OTL
        from oracle.paged_cache import PagedKVCache as OPC
        torch.set_num_threads(os.cpu_count() or 1)
        torch.manual_seed(0)
        pr = w.pair
        mk = (lambda c: OTG(OMC(vocab_size=pr.vocab, **c))) if pr.kind == "gpt" else \
            (lambda c: OTL(OLC(vocab_size=pr.vocab, **c)))
        od, ot = mk(pr.draft).eval(), mk(pr.target).eval()

        def ocache(m):
            c = m.cfg
            per = w.prompt_hi + w.max_new_tokens + w.k + 2
            return OPC(c.n_layers, getattr(c, "n_kv_heads", c.n_heads), c.d_model // c.n_heads, w.block_size,
                       n * ((per + w.block_size - 1) // w.block_size) + 8)

        oreqs = [OS.Request(f"c{i}", p, w.max_new_tokens) for i, p in enumerate(prompts)]
        g = torch.Generator().manual_seed(0)
        t0 = time.perf_counter()
        ores = OS.run_continuous_speculative_batches(od, ot, oreqs, ocache(od), ocache(ot), w.max_batch_size,
                                                     k=w.k, temperature=w.temperature, generator=g)
        csecs = time.perf_counter() - t0
        ctoks = sum(len(r.output_ids) for r in ores) - sum(len(p) for p in prompts)
        cpu = {"value": ctoks / csecs, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"the whole {w.name} workload ({n} requests), fp32 oracle port"}
    res = {"metric": "committed tokens/s (scheduler, whole workload)", "workload": w.name, "k": w.k,
           "temperature": w.temperature, "requests": n_all, "n_gpus": world, "max_batch_size": batch,
           "pool": (f"{args.pool_gb:g} GB of target K/V ({pool_blocks} blocks of {w.block_size} tokens per cache)"
                    if pool_blocks else "sized to the workload's prompts"),
           "step": "reference structure" if args.reference_structure else "default (bonus deferred)",
           "bookkeeping": "host" if args.sched_host_loop else "device",
           "untimed_warm_run": warm,
           "mode": {"spec": "speculative, independent draft", "self": "speculative, draft = target",
                    "plain": "plain continuous batching, no speculation"}[args.sched_mode],
           "generated_tokens": toks, "seconds": secs, "value": toks / secs, "unit": "tokens/s",
           "timing": "CUDA events from the first launch to the last; max over ranks",
           "per_rank": per_rank, "cpu_baseline": cpu}
    if emit and rank == 0:
        print(json.dumps(res), flush=True)
    return res


def micro_prefix(args, device):
    """Prefix caching on a shared-system-prompt workload: the gpt2-small pair,
    N requests (default 256), each prompt a common system prompt
    (--prefix-len tokens, default 512) plus its own suffix of U[16, 128]
    tokens, 64 new tokens, greedy, the whole workload through
    run_continuous_speculative_batches with the prefix index off and on (each
    after an untimed run of the same workload).  Reports committed tokens/s,
    the prompt tokens computed, the index hit rate, and whether both runs gave
    identical outputs."""
    import pse
    from pse import workload as wl
    from pse.scheduler import Request
    w = wl.WORKLOADS["gpt2-small"]
    n = args.rows or 256
    rng = np.random.default_rng(0)
    system = rng.integers(0, w.pair.vocab, size=args.prefix_len).tolist()
    prompts = [system + rng.integers(0, w.pair.vocab, size=int(rng.integers(16, 129))).tolist() for _ in range(n)]
    max_new = 64
    d, t = build_pair(w, torch.bfloat16, device)
    res_by_mode, lines = {}, {}
    for prefix in (False, True):
        for run in ("warm", "timed"):
            reqs = [Request(f"{run}{i}", p, max_new) for i, p in enumerate(prompts)]
            caches = []
            for m in (d, t):
                cfg = m.cfg
                bs = w.block_size
                nb = sum((len(p) + max_new + w.k + 2 + bs - 1) // bs for p in prompts) + 8
                caches.append(pse.PagedKVCache(cfg.n_layers, cfg.n_heads, cfg.d_model // cfg.n_heads, bs, nb,
                                               dtype=torch.bfloat16, device=device, max_requests=n,
                                               prefix_cache=prefix))
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            res = pse.run_continuous_speculative_batches(d, t, reqs, caches[0], caches[1], n, k=w.k)
            torch.cuda.synchronize()
            secs = time.perf_counter() - t0
            if run == "timed":
                by = {r.request_id[len(run):]: r.output_ids for r in res}
                res_by_mode[prefix] = by
                toks = sum(len(by[str(i)]) - len(p) for i, p in enumerate(prompts))
                st = caches[1].prefix.stats() if prefix else None
                computed = sum(len(p) for p in prompts) - (st["hit_tokens"] if st else 0)
                lines[prefix] = {"value": toks / secs, "unit": "tokens/s", "seconds": secs,
                                 "prompt_tokens": sum(len(p) for p in prompts), "prompt_tokens_computed": computed,
                                 "target_index": st}
            del caches, res
            gc.collect()
            torch.cuda.empty_cache()
        # the admission alone: all prompts prefilled in one batched call (after a warm one)
        for run in ("warm", "timed"):
            caches = []
            for m in (d, t):
                cfg = m.cfg
                nb = sum((len(p) + w.block_size - 1) // w.block_size for p in prompts) + 8
                caches.append(pse.PagedKVCache(cfg.n_layers, cfg.n_heads, cfg.d_model // cfg.n_heads, w.block_size,
                                               nb, dtype=torch.bfloat16, device=device, max_requests=n,
                                               prefix_cache=prefix))
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            pse.prefill_requests(d, t, caches[0], caches[1], [f"p{i}" for i in range(n)], prompts)
            torch.cuda.synchronize()
            lines[prefix]["prefill_seconds"] = time.perf_counter() - t0
            del caches
            gc.collect()
            torch.cuda.empty_cache()
    same = res_by_mode[False] == res_by_mode[True]
    print(json.dumps({"metric": "committed tokens/s (scheduler, shared system prompt)", "workload":
                      f"gpt2-small pair, {n} requests: {args.prefix_len}-token system prompt + U[16,128] suffix, "
                      f"{max_new} new, k={w.k}, greedy, bf16", "prefix_cache_off": lines[False],
                      "prefix_cache_on": lines[True], "speedup": lines[True]["value"] / lines[False]["value"],
                      "prefill_speedup": lines[False]["prefill_seconds"] / lines[True]["prefill_seconds"],
                      "outputs_identical": same}), flush=True)


def micro_tree(args, device):
    """Token-tree speculation against the linear chain on the gpt2-small pair,
    bf16, greedy, 256 requests x 64 new tokens through the scheduler (host
    bookkeeping for both, so only the step differs).  Random-init weights make
    an independent draft agree with the target almost never, so the draft
    here is the target with Gaussian noise of --tree-noise x each weight's
    standard deviation added: it agrees often but not always, the regime
    where a second candidate pays.  Reports committed tokens/s and tokens per
    step for k=4 with 1 (linear), 2 and 4 branches, and how many requests'
    outputs equal the linear run's."""
    import pse
    from pse import workload as wl
    from pse.scheduler import Request
    w = wl.WORKLOADS["gpt2-small"]
    n = args.rows or 256
    prompts = wl.prompts(w, seed=0, n=n)
    max_new, k = 64, 4
    _, t = build_pair(w, torch.bfloat16, device)
    torch.manual_seed(1)
    d = type(t)(t.cfg).eval()
    with torch.no_grad():
        for pd, pt in zip(d.parameters(), t.parameters()):
            pd.copy_(pt + args.tree_noise * pt.float().std() * torch.randn_like(pt))
    outs, lines = {}, {}
    for b in (1, 2, 4):
        # one pair of caches per form, the workload run twice on it: the timed
        # run replays the graphs the untimed one captured (one per batch size)
        dc = cache_for(d, w, n, torch.bfloat16, device, 2 * (k + 2) * b, prompts)
        tc = cache_for(t, w, n, torch.bfloat16, device, 2 * (k + 2) * b, prompts)
        for run in ("warm", "timed"):
            reqs = [Request(f"{run}{i}", p, max_new) for i, p in enumerate(prompts)]
            steps = [0]
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if b == 1:
                res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, n, k=k, defer_bonus=False,
                                                             device_bookkeeping=False,
                                                             on_step=lambda ids, r: steps.__setitem__(0, steps[0] + 1))
            else:
                res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, n, k=k, tree_branches=b,
                                                             on_step=lambda ids, r: steps.__setitem__(0, steps[0] + 1))
            torch.cuda.synchronize()
            secs = time.perf_counter() - t0
            if run == "timed":
                by = {r.request_id[len(run):]: r.output_ids for r in res}
                toks = sum(len(by[str(i)]) - len(p) for i, p in enumerate(prompts))
                outs[b] = by
                lines[b] = {"value": toks / secs, "unit": "tokens/s", "seconds": secs, "steps": steps[0],
                            "tokens_per_row_step": toks / max(1, steps[0]) / n}
            del res
        del dc, tc
        gc.collect()
        torch.cuda.empty_cache()
    print(json.dumps({"metric": "committed tokens/s (scheduler, token-tree speculation)", "workload":
                      f"gpt2-small pair, {n} requests x {max_new} new, k={k}, greedy, bf16, draft = target + "
                      f"{args.tree_noise:g} sd noise", "linear": lines[1], "branches_2": lines[2],
                      "branches_4": lines[4],
                      "requests_identical_to_linear": {f"branches_{b}": sum(outs[b][r] == outs[1][r] for r in outs[1])
                                                       for b in (2, 4)},
                      "note": "bf16: the verify call's width differs between the forms (k vs b*k nodes), so a "
                              "near-tie argmax can differ; fp32 parity is exact (tests/test_tree_gpu.py)"}),
          flush=True)


GEMM_SHAPES = {
    # name: (M, K, N, bias, gelu, fp32 out) -- the gpt2-small step's projections
    "t.qkv": (1536, 768, 2304, True, False, False), "t.out": (1536, 768, 768, True, False, False),
    "t.fc1": (1536, 768, 3072, True, True, False), "t.fc2": (1536, 3072, 768, True, False, False),
    "t.lm_head": (1536, 768, 32000, False, False, True),
    "d.qkv": (256, 384, 1152, True, False, False), "d.out": (256, 384, 384, True, False, False),
    "d.fc1": (256, 384, 1536, True, True, False), "d.fc2": (256, 1536, 384, True, False, False),
    "d.lm_head": (256, 384, 32000, False, False, True),
}


def micro_gemm(args, device):
    """The step's projection GEMMs, cuBLAS (torch, bias fused, GELU as a
    separate pass) against pse_gemm_bf16 (tcgen05, bias and GELU fused; as
    dispatched, and with single-CTA tiles only): device us per call (50 calls
    captured in a CUDA graph, replayed 4 times, CUDA events) and TFLOP/s."""
    import pse._native as N
    rows = []
    g = torch.Generator(device=device).manual_seed(0)
    for name, (M, K, Nn, bias, gelu, f32) in GEMM_SHAPES.items():
        if args.gemm_only and name != args.gemm_only:
            continue
        a = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
        w = (torch.randn(Nn, K, device=device, generator=g) * 0.05).to(torch.bfloat16)
        b = torch.randn(Nn, device=device, generator=g).to(torch.bfloat16) if bias else None
        c = torch.empty(M, Nn, device=device, dtype=torch.float32 if f32 else torch.bfloat16)

        def cublas():
            if f32:
                torch.mm(a, w.t(), out_dtype=torch.float32, out=c)
            elif b is not None:
                torch.addmm(b, a, w.t(), out=c)
                if gelu:
                    c.copy_(torch.nn.functional.gelu(c))
            else:
                torch.mm(a, w.t(), out=c)

        def ours():
            N.call("pse_gemm_bf16", a.data_ptr(), K, w.data_ptr(), K, None if b is None else b.data_ptr(),
                   c.data_ptr(), Nn, M, Nn, K, 1 if gelu else 0, 1 if f32 else 0, None, N.stream_ptr())

        def ours_1cta():
            lib = N.load()
            lib.pse_gemm_pair_tiles(0)
            ours()
            lib.pse_gemm_pair_tiles(1)

        if args.gemm_only:  # plain launches of one GEMM only (a short program for ncu)
            for _ in range(max(args.steps, 1)):
                (cublas if args.gemm_impl == "cublas" else ours)()
            torch.cuda.synchronize()
            rows.append({"gemm": name, "M": M, "K": K, "N": Nn, "launches": max(args.steps, 1)})
            continue
        res = {}
        for label, fn in (("cublas", cublas), ("tcgen05", ours), ("tcgen05_1cta", ours_1cta)):
            for _ in range(5):
                fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()  # device time: 50 calls captured, no host dispatch in the timing
            with N.graph_capture(graph):
                for _ in range(50):
                    fn()
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(4):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / 200 * 1000
            res[label] = {"us": round(us, 2), "tflops": round(2 * M * K * Nn / (us * 1e-6) / 1e12, 1)}
        rows.append({"gemm": name, "M": M, "K": K, "N": Nn, **res})
    print(json.dumps({"metric": "projection GEMMs", "rows": rows}), flush=True)


def micro_churn(args, device, emit=True):
    """Truncate churn: 1024 rows of block 16 with lengths U[512, 32768]; each
    step reserves 8 tokens (verify), truncates every row to base + U{0..8}
    and reserves 1 more (bonus), as one step of the engine commits.  1000
    steps, device-resident, replayed from one CUDA graph; reports us/step and
    host syncs per step (0)."""
    import pse
    import pse._native as N
    R, bs, steps = args.rows or 1024, 16, args.steps if args.steps > 30 else 1000
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 32769, size=R)
    nb = int(((lens + 9 * steps + bs) // bs).sum()) + 64
    c = pse.PagedKVCache(1, 1, 1, bs, nb, dtype=torch.float32, device=device, max_requests=R,
                         max_blocks_per_request=int((lens.max() + 9 * steps) // bs + 2))
    slots = torch.arange(R, dtype=torch.int32, device=device)
    base = torch.empty(R, dtype=torch.int32, device=device)
    base2 = torch.empty(R, dtype=torch.int32, device=device)
    st = N.stream_ptr()
    init = torch.from_numpy(lens.astype(np.int32)).to(device)
    # initial lengths: one reserve per distinct length is slow; reserve row by row in one batched call per width
    N.call("pse_kv_reserve", c.state, slots.data_ptr(), R, 0, base.data_ptr(), st)
    for i in range(R):
        N.call("pse_kv_reserve", c.state, slots[i:i + 1].data_ptr(), 1, int(lens[i]), base.data_ptr(), st)
    acc = torch.from_numpy(rng.integers(0, 9, size=(steps, R)).astype(np.int32)).to(device)

    def step(j):
        N.call("pse_kv_reserve", c.state, slots.data_ptr(), R, 8, base.data_ptr(), st)
        N.call("pse_kv_truncate", c.state, slots.data_ptr(), R, None, base.data_ptr(), acc[j].data_ptr(), st)
        N.call("pse_kv_reserve", c.state, slots.data_ptr(), R, 1, base2.data_ptr(), st)

    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with N.graph_capture(g):
        st = N.stream_ptr()
        for j in range(steps):
            step(j)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    status = int(c._blocks.status.item())
    expect = init + (acc.sum(0) + steps).to(torch.int32)
    ok = bool(torch.equal(c._blocks.seq_len[:R], expect)) and status == 0
    res = {"metric": "truncate churn us/step", "value": ms * 1000 / steps, "unit": "us/step",
                      "higher_is_better": False, "rows": R, "block_size": bs, "steps": steps,
                      "host_syncs_per_step": 0, "launches_per_step": 3, "lengths_ok": ok, "status": status,
                      "free_blocks_end": int(c._blocks.free_top.item())}
    if emit:
        print(json.dumps(res), flush=True)
    return res


def kernel_configs(args, device):
    """The kernel microbenchmark configurations, timed after the step on the
    same GPU (each allocates its own buffers): 5a verify attention (1024 rows,
    contexts U[512, 32768], GQA 32/8, head_dim 128, block 16; ~70 GB of K/V),
    5b accept / resample (1024 rows x 8 drafts, vocab 128256, T = 1 and
    T = 0), 5c truncate churn (1024 rows, 1000 steps).  Summaries only."""
    import copy
    gc.collect()
    torch.cuda.empty_cache()
    out = {}
    a = copy.copy(args)
    a.rows, a.steps, a.warmup = None, 10, 3
    a.attn_shape, a.prefill_kernel, a.attn_pages = "verify-5a", "tc", "permuted"
    r = micro_attention(a, device, emit=False)
    out["5a_verify_attention"] = {k: r[k] for k in ("value", "unit", "frac_of_peak", "peak_kind", "us_per_launch",
                                                    "algorithmic_bytes", "rows", "ctx_mean")}
    gc.collect()
    torch.cuda.empty_cache()
    for T in (1.0, 0.0):
        a.temperature, a.accept_kernel = T, 0
        r = micro_accept(a, device, emit=False)
        out[f"5b_accept_T{T:g}"] = {k: r[k] for k in ("value", "unit", "frac_of_peak", "us_per_launch",
                                                     "bytes_needed", "formula_GBps", "mean_accepted", "kernel")}
        gc.collect()
        torch.cuda.empty_cache()
    a.steps = 1000
    r = micro_churn(a, device, emit=False)
    out["5c_truncate_churn"] = {k: r[k] for k in ("value", "unit", "host_syncs_per_step", "lengths_ok", "rows",
                                                  "steps")}
    gc.collect()
    torch.cuda.empty_cache()
    if args.workload == "gpt2-small":
        # every decode position, not only the early steps the replays time: the whole workload
        # (256 requests x 256 new tokens, batched prefill included) through the scheduler
        a.workload, a.rows, a.sched_mode, a.reference_structure = "gpt2-small", None, "spec", False
        a.sched_host_loop, a.no_cpu_baseline = False, True
        r = micro_scheduler(a, device, emit=False)
        out["3_whole_workload"] = {k: r[k] for k in ("value", "unit", "seconds", "generated_tokens", "requests",
                                                     "step", "bookkeeping")}
        gc.collect()
        torch.cuda.empty_cache()
    return out


def llama_whole(args, device):
    """The Llama-style configuration as specified: all 2048 requests through
    the scheduler on this GPU (batched prefill and every decode step), the
    pools sized to ~150 GB of the target's K/V (less if the GPU has less
    free), at most 1024 requests in flight (2048 prompts' K/V would not fit
    150 GB).  One run, graph captures inside the timed region."""
    import copy
    gc.collect()
    torch.cuda.empty_cache()
    free = torch.cuda.mem_get_info(device)[0] / 1e9
    a = copy.copy(args)
    a.workload, a.rows, a.sched_mode, a.reference_structure = "llama-1b", None, "spec", False
    a.sched_host_loop, a.no_cpu_baseline = False, True
    a.max_batch, a.pool_gb = 1024, float(min(150.0, int(free * 0.94 - 14.0)))
    r = micro_scheduler(a, device, emit=False, warm=False)
    gc.collect()
    torch.cuda.empty_cache()
    return {k: r[k] for k in ("value", "unit", "seconds", "generated_tokens", "requests", "max_batch_size", "pool",
                              "step", "bookkeeping", "untimed_warm_run")}


def llama_step(args, device, peak):
    """The Llama-style configuration's step on this GPU (512 rows of its
    workload, bf16, k=4, block 32): the same measurement as the headline on a
    second workload, summarised."""
    import copy
    gc.collect()
    torch.cuda.empty_cache()
    a = copy.copy(args)
    a.workload, a.rows, a.steps, a.warmup = "llama-1b", 512, 10, 3
    a.reference_structure = False
    r = run_pse(a, 0, 1, device)
    hd_, rf_ = r["head"], r["ref"]
    value = hd_["committed"] / (hd_["ms"] / 1000.0)
    achieved = r["attn_bytes"] / (r["attn_ms"] / 1000.0) / 1e9
    roof = (hd_["committed"] / a.steps) / (r["step_bytes"] / (peak * 1e9))
    out = {"workload": "llama-1b: 512 rows (prompts lognormal median 2048, clipped to [128, 8192]), k=4, block 32, "
                       "greedy, bf16", "value": value, "unit": "tokens/s", "ms_per_step": hd_["ms"] / a.steps,
           "e2e": hd_["e2e_tokens"] / (hd_["e2e_ms"] / 1000.0),
           "reference_structure": rf_["committed"] / (rf_["ms"] / 1000.0),
           "verify_attention_frac": achieved / peak, "step_roofline_frac": value / roof,
           "prefill_tokens_per_s": r["prefill_tokens"] / r["prefill_s"], "clocks": r["clocks"]}
    del r
    gc.collect()
    torch.cuda.empty_cache()
    return out


def self_draft_step(args, device):
    """The headline workload's step with draft = target (the reference
    benchmark's ceiling configuration): every draft is accepted, so the timed
    steps commit k+1 tokens per row and exercise multi-token commits, multi-block
    truncation and the all-accepted bonus path that the independent random draft
    almost never reaches.  Summarised."""
    import copy
    gc.collect()
    torch.cuda.empty_cache()
    a = copy.copy(args)
    a.steps, a.warmup, a.self_draft, a.reference_structure = 10, 3, True, False
    r = run_pse(a, 0, 1, device)
    hd_, rf_ = r["head"], r["ref"]
    out = {"workload": f"{args.workload}, draft = target", "value": hd_["committed"] / (hd_["ms"] / 1000.0),
           "unit": "tokens/s", "ms_per_step": hd_["ms"] / a.steps,
           "e2e": hd_["e2e_tokens"] / (hd_["e2e_ms"] / 1000.0),
           "reference_structure": rf_["committed"] / (rf_["ms"] / 1000.0),
           "acceptance": {"rows_by_drafts_accepted": r["acc_hist"], "k": r["k"]}}
    del r
    gc.collect()
    torch.cuda.empty_cache()
    return out


def config_block(args, w, B, world):
    dist = (f"lognormal(median {w.lognormal_median:g}, sigma {w.lognormal_sigma:g}) clipped to "
            f"[{w.prompt_lo},{w.prompt_hi}]" if w.lognormal_sigma > 0 else f"U[{w.prompt_lo},{w.prompt_hi}]")
    return {"workload": f"{w.name}: {w.n_requests if args.rows is None else B} rows/GPU, prompts "
                        f"{dist}, k={w.k}, block {w.block_size}, "
                        f"{'greedy' if w.temperature == 0 else 'T=%g' % w.temperature}",
            "rows_per_gpu": B, "k": w.k, "block_size": w.block_size,
            "target": w.pair.target, "draft": w.pair.draft, "vocab": w.pair.vocab,
            "parallelism": f"request shards x{world}",
            "l2": "KV working set per step (GBs) >> 126 MB L2; no flush needed"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="pse", choices=["pse", "reference"])
    ap.add_argument("--workload", default="gpt2-small")
    ap.add_argument("--rows", type=int, default=None)
    ap.add_argument("--k", type=int, default=None, help="draft length (default: the workload's)")
    ap.add_argument("--sched-mode", default="spec", choices=["spec", "self", "plain"],
                    help="--micro scheduler: independent draft, draft = target, or no speculation")
    ap.add_argument("--max-batch", type=int, default=None,
                    help="--micro scheduler: max_batch_size of the scheduler (default: the workload's)")
    ap.add_argument("--pool-gb", type=float, default=None,
                    help="--micro scheduler: size each pool to this many GB of the target's K/V (default: every "
                         "request's own prompt + new tokens)")
    ap.add_argument("--sched-host-loop", action="store_true",
                    help="--micro scheduler: per-row bookkeeping on the host (the reference's loop) instead of "
                         "on the device")
    ap.add_argument("--step-temperature", type=float, default=None,
                    help="sampling temperature of the step (default: the workload's)")
    ap.add_argument("--cpu-rows", type=int, default=8,
                    help="rows of the CPU sample: the reference's CPU step is fastest per token at 4-8 rows "
                         "(padding to the longest row and the O(rows x longest) gather grow faster than the rows)")
    ap.add_argument("--cpu-steps", type=int, default=4)
    ap.add_argument("--cpu-ladder", default=None,
                    help="comma-separated row counts: time the CPU path at each (1 warm-up + --cpu-steps steps) "
                         "and print one JSON line per count, then exit")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernel-configs", action="store_true",
                    help="skip the 5a / 5b / 5c kernel configurations after the step (they run at N=1 only)")
    ap.add_argument("--no-llama-whole", action="store_true",
                    help="skip the Llama-style whole workload (2048 requests, ~150 GB pools, about a minute) among "
                         "the kernel configurations")
    ap.add_argument("--micro", choices=["attn", "accept", "churn", "prefill", "scheduler", "gemm", "prefix", "tree"],
                    default=None,
                    help="kernel microbenchmark instead of the step")
    ap.add_argument("--temperature", type=float, default=1.0, help="--micro accept: temperature")
    ap.add_argument("--prefix-len", type=int, default=512, help="--micro prefix: system prompt tokens")
    ap.add_argument("--tree-noise", type=float, default=0.1,
                    help="--micro tree: draft = target + this many weight standard deviations of noise")
    ap.add_argument("--accept-kernel", type=int, default=0, choices=[0, 1, 2, 3],
                    help="--micro accept at T > 0: 0 cluster-split streaming (default), 1 scalar CTA per row, "
                         "2 cluster per row holding the row on chip, 3 streaming CTA per row")
    ap.add_argument("--reference-structure", action="store_true",
                    help="headline the reference's step structure (2 target calls per step) instead of the "
                         "default step (the target's bonus call deferred into the next verify)")
    ap.add_argument("--attn-shape", default="gpt2-verify", choices=sorted(ATTN_SHAPES))
    ap.add_argument("--gemm-only", default=None, choices=sorted(GEMM_SHAPES),
                    help="--micro gemm: launch only this shape's tcgen05 GEMM, --steps times, without graphs or "
                         "timing (a short program for ncu)")
    ap.add_argument("--gemm-impl", default="tc", choices=["tc", "cublas"],
                    help="--gemm-only: launch the tcgen05 GEMM (tc) or cuBLAS through torch (cublas)")
    ap.add_argument("--prefill-kernel", default="tc", choices=["tc", "off", "single"],
                    help="wide attention calls (prefill) on the tcgen05 kernels, on the mma.sync kernel, or on the "
                         "one-query-tile tcgen05 kernel at every head_dim")
    ap.add_argument("--attn-pages", default="permuted", choices=["permuted", "contiguous"],
                    help="--micro attn: block tables a random permutation of the pool, or consecutive blocks")
    ap.add_argument("--tc-gemm", default=None, choices=["off", "gelu", "all"],
                    help="bf16 projections: cuBLAS (off), the tcgen05 GEMM for the GELU up-projections only (gelu), "
                         "or the tcgen05 GEMM for every projection (all); default: the engine's setting")
    ap.add_argument("--profile-step", action="store_true",
                    help="after warm-up run one eager step inside the NVTX range 'pse_step' and exit (for ncu)")
    args = ap.parse_args()

    from pse import workload as wl
    if args.k is not None or args.step_temperature is not None:  # e.g. the k sweep of the T = 1 workload
        import dataclasses
        w0 = wl.WORKLOADS[args.workload]
        wl.WORKLOADS[args.workload] = dataclasses.replace(
            w0, k=w0.k if args.k is None else args.k,
            temperature=w0.temperature if args.step_temperature is None else args.step_temperature)
    w = wl.WORKLOADS[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric = "committed tokens/s"

    if args.cpu_ladder:
        threads = os.cpu_count() or 1
        for rows in [int(x) for x in args.cpu_ladder.split(",")]:
            r = cpu_reference(args, rows, args.cpu_steps, threads, warmup=1)
            print(json.dumps({"metric": "CPU reference-path committed tokens/s by batch rows", "workload": w.name,
                              "rows": rows, "value": r["value"], "unit": "tokens/s", "seconds": r["seconds"],
                              "cores": r["cores"], "sample": r["sample"]}), flush=True)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        threads = os.cpu_count() or 1
        # each step of this arm is one batched step over a bounded sample of the rows
        r = cpu_reference(args, args.cpu_rows, args.steps, threads, warmup=args.warmup)
        line = {"impl": "reference", "metric": metric, "value": r["value"], "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * r["seconds"] / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic prompts (seeded), random-init weights (seed 0)",
                "config": config_block(args, w, w.max_batch_size if args.rows is None else args.rows, args.gpus),
                "cpu_baseline": {"value": r["value"], "unit": "tokens/s", "cores": r["cores"], "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if world > 1:
        import datetime
        # NCCL's communicator lines (ranks, devices, transports) go to the log
        # (the image's default level, VERSION, prints only the version)
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() in ("", "VERSION", "WARN"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    device = torch.device("cuda", local if world > 1 else torch.cuda.current_device())
    torch.cuda.set_device(device)
    import pse._build
    pse._build.build()
    if args.tc_gemm is not None:
        import pse.engine
        pse.engine.USE_TC_GEMM = {"off": False, "gelu": "gelu", "all": True}[args.tc_gemm]
    if args.micro == "attn":
        micro_attention(args, device)
        return
    if args.micro == "accept":
        micro_accept(args, device)
        return
    if args.micro == "churn":
        micro_churn(args, device)
        return
    if args.micro == "prefill":
        micro_prefill(args, device)
        return
    if args.micro == "scheduler":
        micro_scheduler(args, device)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return
    if args.micro == "prefix":
        micro_prefix(args, device)
        return
    if args.micro == "tree":
        micro_tree(args, device)
        return
    if args.micro == "gemm":
        micro_gemm(args, device)
        return
    r = run_pse(args, rank, world, device)
    if r is None:
        return
    peak, peak_kind = _peaks()
    kernel_cfgs = None
    if world == 1 and not args.no_kernel_configs:
        kernel_cfgs = kernel_configs(args, device)
        if args.workload == "gpt2-small":
            kernel_cfgs["4_llama_1b_step"] = llama_step(args, device, peak)
            if not args.no_llama_whole:
                kernel_cfgs["4_llama_1b_whole_workload"] = llama_whole(args, device)
        kernel_cfgs["self_draft_step"] = self_draft_step(args, device)
    check = token_check(args, r["check_rows"], os.cpu_count() or 1) if rank == 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference(args, args.cpu_rows, args.cpu_steps, os.cpu_count() or 1)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    hd_, rf_ = r["head"], r["ref"]
    value = hd_["committed"] / (hd_["ms"] / 1000.0)
    achieved = r["attn_bytes"] / (r["attn_ms"] / 1000.0) / 1e9
    per_gpu_tok_step = hd_["committed"] / args.steps / world
    roof_tok_s = per_gpu_tok_step / (r["step_bytes"] / (peak * 1e9)) * world
    ratio = ATTN_TRAFFIC_RATIO.get((args.workload, r["attn_width"]))
    line = {
        "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": hd_["ms"] / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if "bfloat16" in r["dtype"] else "f32",
        "data": "synthetic prompts (seeded), random-init weights (seed 0)",
        "config": config_block(args, w, r["B"], world),
        "step": ("default step (target bonus call deferred into the next verify): 1 target call of width k+1 + "
                 "k+1 draft calls per step; tokens, block tables, lengths and free lists identical to the "
                 "reference structure; e2e driven by the reference scheduler's unchanged call "
                 "(returned logits handed back)" if r["deferred"] else
                 "reference structure: 2 target + k+1 draft calls per step"),
        "e2e": {"value": hd_["e2e_tokens"] / (hd_["e2e_ms"] / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
        "reference_structure": {"value": rf_["committed"] / (rf_["ms"] / 1000.0),
                                "ms_per_step": rf_["ms"] / args.steps,
                                "e2e": rf_["e2e_tokens"] / (rf_["e2e_ms"] / 1000.0)},
        "roofline": {"kernel": f"pse_paged_attention (target verify, width {r['attn_width']}, all layers)",
                     "bound": "hbm", "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": achieved / peak,
                     "traffic": None if ratio is None else ratio * r["attn_bytes"],
                     "traffic_note": None if ratio is None else
                     "ncu dram bytes / algorithmic bytes of the same kernel on the gpt2-verify microbench shape, "
                     "scaled to this launch's algorithmic bytes",
                     "avg_launch_us": r["attn_ms"] * 1000, "algorithmic_bytes": r["attn_bytes"]},
        "step_roofline": {"bound": "hbm (KV + weights of 1 target pass of width k+1 and k draft passes)",
                          "bytes_per_step_per_gpu": r["step_bytes"], "tokens_per_step_per_gpu": per_gpu_tok_step,
                          "roofline_tokens_s": roof_tok_s, "frac": value / roof_tok_s},
        "cpu_baseline": None if cpu is None else {"value": cpu["value"], "unit": "tokens/s", "cores": cpu["cores"],
                                                  "kind": "port", "sample": cpu["sample"]},
        "clocks": r["clocks"],
        "gpu_launches": r["kernels_per_step"] * args.steps,
        "token_check": check,
        "kernel_configs": kernel_cfgs,
        "acceptance": {"rows_by_drafts_accepted": r["acc_hist"], "k": r["k"],
                       "note": "rank 0's rows over the timed steps, index = drafts accepted (0..k)"},
        "prefill": {"requests": r["B"], "prompt_tokens": r["prefill_tokens"], "seconds": r["prefill_s"],
                    "tokens_per_s": r["prefill_tokens"] / r["prefill_s"], "mode": "batched (prefill_requests)"},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
