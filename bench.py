#!/usr/bin/env python3
"""bench.py -- accepted tokens/s of 4-bit speculative decoding on B200.

Workloads (--workload):
  qwen3-8b-draft0.6b-k5-bs8-t0.7 (default, configs[2]): Qwen3-8B architecture
    target (36 layers, hidden 4096, 32 q / 8 kv heads, FFN 12288, vocab 151936)
    with a separate Qwen3-0.6B draft (28 layers), both synthetic N(0,0.02)
    weights quantized affine 4-bit group 64 (seeds 2026 / 2027); K = 5;
    8 sequences of 512 uniform-random prompt tokens; 512 new tokens each;
    temperature 0.7, top-p 0.9 rejection sampling; 4-bit group-64 KV cache.
    The verify pass (M = 48) runs the tcgen05 path.
  qwen3-0.6b-selfdraft2-k4-bs1: Qwen3-0.6B target, draft = its
    first 2 layers + shared embedding / lm_head; K = 4; batch 1; 128-token
    prompt; 256 greedy new tokens; bf16 KV cache.
  --qmm-sweep: the op-level quantized_matmul sweep.

A "step" is one generation of the workload through the public API
(lmx_spec_prefill with the prompts in host memory, lmx_spec_decode,
lmx_spec_result reading the tokens back).  value = tokens / decode time
(device events, prefill excluded, the reference's GenerateCompletionInfo
definition); e2e = tokens / wall time of the whole API sequence including the
host<->device copies and the prefill.  One process per GPU; for N > 1 each
rank decodes its own sequences (independent batches, no data-path
collective: weak scaling; bs1 is "replicas only").

--impl reference times the CPU restatement of the reference's algorithm
(oracle/, the reference's MLX CPU backend cannot be built here) on the host
cores with the same weights, prompts and decode loop.
"""
import argparse
import ctypes as C
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# configs[0] (bs1, greedy, self-draft) and configs[2] (bs8, stochastic, separate
# Qwen3-0.6B draft over a Qwen3-8B target, 4-bit KV).  `cpu_prompt` shortens
# the prompt of the bounded CPU sample only (its prefill is untimed).
WORKLOADS = {
    "qwen3-0.6b-selfdraft2-k4-bs1": dict(arch="QWEN3_0_6B", draft=None, draft_layers=2, K=4,
                                         batch=1, prompt=128, new=256, kv_bits=16,
                                         temperature=0.0, top_p=1.0, cpu_prompt=None,
                                         profile="verify_pass_qwen3_0.6b_k4_bs1.md"),
    "qwen3-8b-draft0.6b-k5-bs8-t0.7": dict(arch="QWEN3_8B", draft="QWEN3_0_6B", draft_layers=28,
                                           K=5, batch=8, prompt=512, new=512, kv_bits=4,
                                           temperature=0.7, top_p=0.9, cpu_prompt=32, cpu_steps=3, steps=5,
                                           profile="verify_pass_qwen3_8b_k5_bs8.md"),
    # Qwen3-Next-style hybrid (Gated DeltaNet : gated attention
    # 3:1, 512 experts top-10 + shared expert) with its MTP head drafting 2
    # tokens; replicas only (each rank decodes its own 4 sequences).
    "qwen3-next-mtp2-bs4": dict(arch="QWEN3_NEXT_HYBRID", hybrid=True, K=2, batch=4, prompt=1024, new=128,
                                kv_bits=16, temperature=0.0, top_p=1.0, steps=2, draft=None,
                                draft_layers=0, profile="verify_pass_qwen3_next_mtp2_bs4.md"),
    # tensor-parallel over the N GPUs (strong scaling); the draft
    # runs replicated on every rank.  The 8192-token random prefix is an
    # 8160-row synthetic KV context plus a 32-token random prompt.
    "llama3-70b-draft1b-k4-bs16-ctx8k-tp": dict(arch="LLAMA3_70B", draft="LLAMA32_1B", draft_layers=16,
                                                K=4, batch=16, prompt=32, context=8160, new=64, kv_bits=8,
                                                temperature=0.0, top_p=1.0, cpu_prompt=None, steps=3,
                                                tp=True, profile="verify_pass_llama3_70b_k4_bs16.md"),
}
DEFAULT_WORKLOAD = "qwen3-8b-draft0.6b-k5-bs8-t0.7"
METRIC = "accepted tokens/s (4-bit spec decode, bs1/bs8); verify-pass HBM GB/s vs 8 TB/s"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            v = [x.strip() for x in line.split(",")]
            if len(v) < 9:
                continue
            try:
                sm.append(float(v[1]))
                mx = float(v[2])
            except ValueError:
                continue
            for n, flag in zip(names, v[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local}"))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch
        import torch.distributed as dist
        dist.barrier()
        torch.cuda.synchronize()


def reduce(world, vals, op="max"):
    if world == 1:
        return vals
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return t.tolist()


def cpu_sample(wl, prompts, lmx_cfg, draft_cfg, seed, steps, warmup):
    """Time the oracle's decode loop on the host cores (prefill untimed).
    The oracle runs every quantized matmul in its canonical order (the
    reference's affine identity, its fastest CPU form)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    L = O.lib()

    def create(c, sd):
        cfg = dict(c)
        cfg["group"] = cfg.pop("group_size")
        return L.orc_model_create(C.byref(O.ModelCfg(**cfg)), sd)

    L.orc_set_mma_min_m(0)
    L.orc_set_threads(0)  # every host core, whatever OMP_NUM_THREADS the launcher exported
    t0 = time.time()
    model = create(lmx_cfg, seed)
    dmodel = create(draft_cfg, seed + 1) if draft_cfg else None
    setup = time.time() - t0
    # cpu_prompt: the sample prefills only the last cpu_prompt prompt tokens
    # through the model; the rows before them are a seeded synthetic KV
    # context, so the timed decode reads a cache of the workload's length
    cp = wl["cpu_prompt"] or prompts.shape[1]
    ctx = prompts.shape[1] - cp
    prm = O.SpecParams(K=wl["K"], max_tokens=wl["new"], temperature=wl["temperature"],
                       top_p=wl["top_p"], seed=seed, draft_layers=wl["draft_layers"],
                       context_len=ctx, context_seed=seed)
    p = np.ascontiguousarray(prompts[:, prompts.shape[1] - cp:], dtype=np.int32)
    ss = L.orc_spec_session(model, dmodel, O.ptr(p), p.shape[0], p.shape[1], prm, wl["kv_bits"])
    st = np.zeros(5, np.int64)
    L.orc_spec_session_step(ss, warmup)
    L.orc_spec_session_result(ss, None, O.ptr(st))
    e0, t0 = int(st[3]), time.perf_counter()
    n = L.orc_spec_session_step(ss, steps)
    dt = time.perf_counter() - t0
    L.orc_spec_session_result(ss, None, O.ptr(st))
    tokens = int(st[3]) - e0
    L.orc_spec_session_free(ss)
    L.orc_model_free(model)
    if dmodel:
        L.orc_model_free(dmodel)
    L.orc_set_mma_min_m(16)
    return dict(value=tokens / dt if dt > 0 else 0.0, tokens=tokens, seconds=dt, spec_steps=n,
                cores=L.orc_threads(), prefill_s=st[4] * 1e-9, setup_s=setup, prompt=p.shape[1], context=ctx)


def cpu_sample_text(r, steps):
    pre = (f"a {r['context']}-row synthetic KV context + a {r['prompt']}-token prompt prefill (untimed) in place "
           f"of the {r['context'] + r['prompt']}-token prompt" if r["context"] else
           f"an untimed {r['prompt']}-token prefill")
    return (f"{steps} speculative steps ({r['tokens']} tokens) of the workload's decode after {pre}; "
            f"oracle/ C++ restatement, canonical order, {r['cores']} threads")


def cpu_sample_composed(wl, arch, darch, seed, reps, tokens_per_step):
    """Bounded CPU sample of a workload too large for the host (configs[4]:
    80 layers of 8192-wide weights): the oracle times one decoder layer of
    the full-size target at the verify shape (M = B(K+1)) over the full
    synthetic context, with and without its lm_head, and the same for one
    draft layer at M = B; a speculative step is composed as
    L_t * layer_t + head_t + K (L_d * layer_d + head_d), and tokens/s =
    tokens_per_step * B / step."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    L = O.lib()
    L.orc_set_mma_min_m(0)
    L.orc_set_threads(0)  # every host core, whatever OMP_NUM_THREADS the launcher exported
    B, K, ctx = wl["batch"], wl["K"], wl.get("context", 0) + wl["prompt"]
    rng = np.random.RandomState(seed)

    def layer_times(c, T, sd, tid_base):
        cfg = dict(c, layers=1)
        cfg["group"] = cfg.pop("group_size")
        m = L.orc_model_create(C.byref(O.ModelCfg(**cfg)), sd)
        oc = L.orc_cache_create(m, 1, B, ctx + (2 * reps + 2) * T + 8, wl["kv_bits"])
        L.orc_cache_fill_synthetic(oc, ctx, seed, tid_base)
        logits = np.zeros((B, T, c["vocab"]), np.uint16)
        out = []
        for with_head in (False, True):
            for i in range(reps + 1):  # the first forward is warm-up
                tok = rng.randint(0, c["vocab"], (B, T)).astype(np.int32)
                t0 = time.perf_counter()
                L.orc_forward(m, oc, 1, O.ptr(tok), B, T, O.ptr(logits) if with_head else None)
                dt = time.perf_counter() - t0
                if i:
                    out.append((with_head, dt))
        L.orc_cache_free(oc)
        L.orc_model_free(m)
        body = statistics.median([d for h, d in out if not h])
        head = max(0.0, statistics.median([d for h, d in out if h]) - body)
        return body, head

    t0 = time.time()
    tl, th = layer_times(arch, K + 1, seed, 0x40000000)
    dl, dh = layer_times(darch, 1, seed + 1, 0x50000000)
    step = arch["layers"] * tl + th + K * (wl["draft_layers"] * dl + dh)
    L.orc_set_mma_min_m(16)
    return dict(value=tokens_per_step * B / step, step_s=step, layer_s=tl, head_s=th, dlayer_s=dl,
                dhead_s=dh, cores=L.orc_threads(), wall_s=time.time() - t0)


def cpu_sample_hybrid(wl, arch, seed, reps, tokens_per_step):
    """Bounded CPU sample of configs[3]: the oracle times a 2-layer model
    (one Gated DeltaNet + one gated-attention layer, each with its MoE block)
    of the full widths at the verify shape (B x 3 tokens over the prompt's
    cache), with and without the lm_head; the oracle's MoE cost is per
    (token, selected expert), so 16 experts stand in for 512 (the router is
    timed separately at full width).  A step = 24 x the 2-layer body + head
    + 2 MTP drafts (each one attention + MoE layer on B rows + head)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    L = O.lib()
    L.orc_set_mma_min_m(0)
    L.orc_set_threads(0)  # every host core, whatever OMP_NUM_THREADS the launcher exported
    B, P = wl["batch"], wl["prompt"]
    cfg = dict(arch, layers=2, attn_every=2, experts=max(16, arch["top_k"] + 1))
    t0 = time.time()
    m = L.orc_hybrid_create(C.byref(O.HybridCfg(**cfg)), seed)
    rng = np.random.RandomState(seed)
    st = L.orc_hybrid_state_create(m, B, P + 64, wl["kv_bits"])
    pre = rng.randint(0, arch["vocab"], (B, 32)).astype(np.int32)
    L.orc_hybrid_forward(m, st, O.ptr(pre), B, 32, None)
    lg = np.zeros((B, 3, arch["vocab"]), np.uint16)
    body, full = [], []
    for i in range(reps + 1):
        tok = rng.randint(0, arch["vocab"], (B, 3)).astype(np.int32)
        a = time.perf_counter()
        L.orc_hybrid_forward(m, st, O.ptr(tok), B, 3, None)
        b_ = time.perf_counter()
        L.orc_hybrid_forward(m, st, O.ptr(tok), B, 3, O.ptr(lg))
        c_ = time.perf_counter()
        if i:
            body.append(b_ - a)
            full.append(c_ - b_)
    L.orc_hybrid_state_free(st)
    L.orc_hybrid_free(m)
    L.orc_set_mma_min_m(16)
    t2 = statistics.median(body)
    head = max(0.0, statistics.median(full) - t2)
    # the cached context is 32 tokens here, not 1024: attention is a small
    # share of the per-layer cost (experts and projections dominate)
    step = (arch["layers"] / 2) * t2 + head + 2 * (t2 / 2 + head)
    return dict(value=tokens_per_step * B / step, step_s=step, body_s=t2, head_s=head, cores=L.orc_threads(),
                wall_s=time.time() - t0)


def run_hybrid(args, wl, world, rank, local):
    """configs[3] through the public hybrid API (lmx_hybrid_spec_*)."""
    lmx = _load("lmx", os.path.join(ROOT, "lemon-mlx-engine_b200", "lmx.py"))
    lmx.call("lmx_set_device", local)
    arch = getattr(lmx, wl["arch"])
    if args.layers:
        arch = dict(arch, layers=args.layers)
    B, P, MT = wl["batch"], wl["prompt"], wl["new"]
    # N > 1: expert parallelism (every rank decodes the same B sequences with
    # its 1/N of the experts; strong scaling); --replicas: independent copies
    ep = world > 1 and not args.replicas
    comm = None
    h = C.c_void_p()
    if ep:
        comm = lmx.TpComm.from_process_group(max_rows=B * 32 * arch["top_k"], max_hidden=arch["hidden"])
        lmx.call("lmx_hybrid_create_ep", C.byref(lmx.HybridConfig(**arch)), args.seed, comm.h, C.byref(h))
    else:
        lmx.call("lmx_hybrid_create", C.byref(lmx.HybridConfig(**arch)), args.seed, C.byref(h))
    sp = C.c_void_p()
    lmx.call("lmx_hybrid_spec_create", h, B, MT, P, wl["kv_bits"], C.byref(sp))
    prompts = np.random.RandomState(args.seed + (rank if world > 1 and not ep else 0)).randint(
        0, arch["vocab"], (B, P)).astype(np.int32)
    out = np.zeros((B, MT), np.int32)
    stats = np.zeros(5, np.int64)

    def one():
        t0 = time.perf_counter()
        lmx.call("lmx_hybrid_spec_prefill", sp, prompts.ctypes.data)
        sec = C.c_double()
        lmx.call("lmx_hybrid_spec_decode", sp, 1, C.byref(sec))
        lmx.call("lmx_hybrid_spec_result", sp, out.ctypes.data, stats.ctypes.data)
        return time.perf_counter() - t0, sec.value, stats.copy()

    if args.profile_verify:
        # prefill only, then N verify passes inside the NVTX range lmx_verify_pass
        lmx.call("lmx_hybrid_spec_prefill", sp, prompts.ctypes.data)
        vs, vb = C.c_double(), C.c_double()
        lmx.call("lmx_hybrid_spec_profile", sp, args.profile_verify, C.byref(vs), C.byref(vb))
        print(json.dumps({"verify_pass_us": round(vs.value * 1e6, 2), "bytes": vb.value}), flush=True)
        lmx.lib().lmx_hybrid_spec_free(sp)
        lmx.lib().lmx_hybrid_free(h)
        if comm is not None:
            barrier(world)
            comm.close()
        return 0
    for _ in range(args.warmup):
        one()
    clocks = Clocks(local)
    barrier(world)
    launches0 = lmx.lib().lmx_launch_count()
    clocks.start()
    wall, dec, toks, acc, prop, steps, replays = 0.0, 0.0, 0, 0, 0, 0, 0
    for _ in range(args.steps):
        w, d, st = one()
        wall += w
        dec += d
        toks += min(int(st[3]), B * MT)
        steps += int(st[0])
        prop += int(st[1])
        acc += int(st[2])
        replays += int(st[4])
    barrier(world)
    ck = clocks.stop()
    nl = C.c_int64()
    lmx.call("lmx_hybrid_spec_step_launches", sp, C.byref(nl))
    gpu_launches = lmx.lib().lmx_launch_count() - launches0 + replays * nl.value
    vsec, vbytes = C.c_double(), C.c_double()
    lmx.call("lmx_hybrid_spec_profile", sp, 10, C.byref(vsec), C.byref(vbytes))
    vsec, vbytes = vsec.value, vbytes.value
    wall_m, dec_m = reduce(world, [wall, dec], "max")
    # expert parallelism: every rank emits the same tokens
    toks_all = toks if ep else int(reduce(world, [float(toks)], "sum")[0])
    peak, peak_kind = peaks()
    achieved = vbytes / vsec / 1e9
    par = (f"ep{world} (experts sharded, {arch['experts'] // world} per rank; the rest replicated)" if ep
           else (f"replicas x{world} (independent sequences per rank)" if world > 1 else "1 GPU"))
    res = {
        "metric": METRIC, "value": round(toks_all / dec_m, 3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * wall_m / args.steps, 3), "higher_is_better": True,
        "scaling": "strong" if ep else "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "batch": B, "prompt": P, "new_tokens": MT, "kv_bits": wl["kv_bits"],
                   "weights": "4-bit g64", "draft": "MTP head, 2 tokens per step", "temperature": 0.0,
                   "parallelism": par,
                   "l2": f"weights and experts ({vbytes / 1e6:.0f} MB per verify pass) exceed L2; no flush"},
        "e2e": {"value": round(toks_all / wall_m, 3), "unit": "tokens/s",
                "h2d_bytes_per_step": B * P * 4, "d2h_bytes_per_step": B * MT * 4 + 40},
        "roofline": {"bound": "hbm", "kernel": f"verify pass ({arch['layers']} layers + lm_head, {B * 3} rows"
                                               + (f", per rank of ep{world})" if ep else ")"),
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_source": peak_kind, "algorithmic_bytes": vbytes, "verify_pass_us": round(vsec * 1e6, 2),
                     "traffic": None},
        "acceptance": {"accepted": acc, "proposed": prop, "rate": round(acc / prop, 4) if prop else None,
                       "tokens_per_step": round(toks / max(1, steps), 3)},
        "clocks": ck, "gpu_launches": int(gpu_launches),
    }
    if world == 1 and rank == 0 and not args.no_cpu:
        tps = toks / max(1, steps)
        r = cpu_sample_hybrid(wl, arch, args.seed, 2, tps)
        res["cpu_baseline"] = {"value": round(r["value"], 4), "unit": "tokens/s", "cores": r["cores"], "kind": "port",
                               "sample": cpu_hybrid_sample_text(wl, arch, r, tps)}
    if rank == 0:
        print(json.dumps(res), flush=True)
    lmx.lib().lmx_hybrid_spec_free(sp)
    lmx.lib().lmx_hybrid_free(h)
    if comm is not None:
        barrier(world)
        comm.close()
    return 0


def cpu_hybrid_sample_text(wl, arch, r, tps):
    return (f"oracle/ C++ restatement, {r['cores']} threads: a 2-layer slice (one Gated DeltaNet + one gated "
            f"attention layer, full widths, 16 experts for the per-token expert cost) at {wl['batch']} x 3 verify "
            f"rows ({r['body_s'] * 1e3:.0f} ms) x {arch['layers'] // 2} + lm_head ({r['head_s'] * 1e3:.0f} ms) + 2 "
            f"MTP drafts = {r['step_s']:.2f} s per step at {tps:.3f} tokens per sequence-step "
            f"({r['wall_s']:.0f} s of CPU sampling)")


def cpu_composed_sample_text(wl, arch, r, tps):
    return (f"oracle/ C++ restatement, {r['cores']} threads: one full-size target layer at "
            f"M={wl['batch'] * (wl['K'] + 1)} over a {wl['context'] + wl['prompt']}-row context "
            f"({r['layer_s'] * 1e3:.0f} ms) x {arch['layers']} + lm_head ({r['head_s'] * 1e3:.0f} ms) + "
            f"K={wl['K']} x (draft layer {r['dlayer_s'] * 1e3:.0f} ms x {wl['draft_layers']} + draft head "
            f"{r['dhead_s'] * 1e3:.0f} ms) = {r['step_s']:.2f} s per step at {tps:.3f} tokens per "
            f"sequence-step ({r['wall_s']:.0f} s of CPU sampling)")


def run_reference(args, wl, world, rank):
    if rank != 0:
        return 0
    lmx = _load("lmx", os.path.join(ROOT, "lemon-mlx-engine_b200", "lmx.py"))
    arch = getattr(lmx, wl["arch"])
    darch = getattr(lmx, wl["draft"]) if wl["draft"] else None
    prompts = np.random.RandomState(args.seed).randint(0, arch["vocab"], (wl["batch"], wl["prompt"]))
    if wl.get("hybrid"):
        r = cpu_sample_hybrid(wl, arch, args.seed, max(1, args.steps), 1.0)
        line = {
            "impl": "reference", "metric": METRIC, "value": round(r["value"], 4), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * r["step_s"], 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "batch": wl["batch"], "prompt": wl["prompt"],
                       "new_tokens": wl["new"], "kv_bits": wl["kv_bits"]},
            "cpu_baseline": {"value": round(r["value"], 4), "unit": "tokens/s", "cores": r["cores"], "kind": "port",
                             "sample": cpu_hybrid_sample_text(wl, arch, r, 1.0)},
            "e2e": {"value": round(r["value"], 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    if wl.get("tp"):
        # composed sample; a step emits at least one token per sequence (the
        # lower bound is used: no device run here to measure acceptance)
        r = cpu_sample_composed(wl, arch, darch, args.seed, max(1, args.steps), 1.0)
        line = {
            "impl": "reference", "metric": METRIC, "value": round(r["value"], 4), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * r["step_s"], 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "batch": wl["batch"], "K": wl["K"],
                       "prompt": wl["prompt"], "context": wl["context"] + wl["prompt"],
                       "new_tokens": wl["new"], "kv_bits": wl["kv_bits"]},
            "cpu_baseline": {"value": round(r["value"], 4), "unit": "tokens/s", "cores": r["cores"],
                             "kind": "port", "sample": cpu_composed_sample_text(wl, arch, r, 1.0)},
            "e2e": {"value": round(r["value"], 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    # each timed step is one speculative step of the same decode (bounded sample)
    r = cpu_sample(wl, prompts, arch, darch, args.seed, args.steps, args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["value"], 3), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * r["seconds"] / max(1, r["spec_steps"]), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": args.workload, "batch": wl["batch"], "K": wl["K"],
                   "prompt": wl["prompt"], "new_tokens": wl["new"], "kv_bits": wl["kv_bits"]},
        "cpu_baseline": {"value": round(r["value"], 3), "unit": "tokens/s", "cores": r["cores"],
                         "kind": "port",
                         "sample": cpu_sample_text(r, args.steps)},
        "e2e": {"value": round(r["value"], 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_lmx(args, wl, world, rank, local):
    lmx = _load("lmx", os.path.join(ROOT, "lemon-mlx-engine_b200", "lmx.py"))
    lmx.call("lmx_set_device", local)
    if args.sdpa_tc_min_cache >= 0:
        lmx.call("lmx_set_sdpa_tc_min_cache", args.sdpa_tc_min_cache)
    if args.gemm_tcs_max_m >= 0:
        lmx.call("lmx_set_gemm_tcs_max_m", args.gemm_tcs_max_m)
    arch = getattr(lmx, wl["arch"])
    if args.layers:
        arch = dict(arch, layers=args.layers)
    darch = getattr(lmx, wl["draft"]) if wl["draft"] else None
    tp = bool(wl.get("tp"))
    B_all, P, ctx = wl["batch"], wl["prompt"], wl.get("context", 0)
    # data parallel: the workload's B sequences are split over
    # the ranks (rank r decodes global sequences [b0, b1)), total work fixed;
    # --replicas (or a batch smaller than the world) gives every rank its own
    # B sequences instead (weak scaling)
    split = not tp and world > 1 and not args.replicas and B_all >= world
    b0, b1 = (rank * B_all // world, (rank + 1) * B_all // world) if split else (0, B_all)
    B = b1 - b0
    comm = None
    if tp and world > 1:  # one shard per rank; handles exchanged over the process group
        comm = lmx.TpComm.from_process_group(max_rows=B * 32, max_hidden=arch["hidden"])
    target = lmx.Model(arch, args.seed, comm=comm)
    # separate draft model (seed + 1) or the target's first layers (self-draft)
    # tensor parallel: the draft is this rank's shard over the same
    # communicator (--replicated-draft: a whole copy on every rank)
    shard_draft = comm is not None and darch is not None and not args.replicated_draft
    draft = lmx.Model(darch, args.seed + 1, comm=comm if shard_draft else None) if darch else None
    # one seeded prompt array for the whole job (split: this rank's slice of
    # it; tensor parallel: all of it on every rank); replicas: per-rank seeds
    replicas = not tp and world > 1 and not split
    prompts = np.random.RandomState(args.seed + (rank if replicas else 0)).randint(
        0, arch["vocab"], (B_all, P)).astype(np.int32)[b0:b1]
    sd = lmx.SpecDecoder(target, draft, wl["draft_layers"], B, wl["K"], wl["new"], P,
                         kv_bits=wl["kv_bits"], temperature=wl["temperature"], top_p=wl["top_p"],
                         seed=args.seed, context_len=ctx, context_seed=args.seed, seq_base=b0)

    if args.profile_verify or args.profile_draft:
        # prefill only (KV cache at the prompt length), then N verify passes
        # (NVTX range lmx_verify_pass) or N single-token draft forwards
        # (lmx_draft_token)
        sd.prefill(prompts)
        if args.profile_verify:
            sd.profile(0, args.profile_verify)
        else:
            sd.profile(1, args.profile_draft)
        sd.close()
        target.close()
        if comm is not None:
            barrier(world)
            comm.close()
        return 0

    def one():
        t0 = time.perf_counter()
        sd.prefill(prompts)
        dsec = sd.decode(use_graph=True)
        out, st = sd.result()
        return time.perf_counter() - t0, dsec, out, st

    for _ in range(args.warmup):
        one()
    clocks = Clocks(local)
    barrier(world)
    launches0 = lmx.lib().lmx_launch_count()
    clocks.start()
    wall, dec, toks, acc, prop, steps, replays = 0.0, 0.0, 0, 0, 0, 0, 0
    for _ in range(args.steps):
        w, d, out, st = one()
        wall += w
        dec += d
        toks += min(st["emitted"], B * wl["new"])
        acc += st["accepted"]
        prop += st["proposed"]
        steps += st["steps"]
        replays += st["replays"]
    barrier(world)
    ck = clocks.stop()
    # eager launches (prefill) counted by the library + graph replays x the
    # kernels captured in one step
    gpu_launches = lmx.lib().lmx_launch_count() - launches0 + replays * sd.step_launches()
    # verify-pass and lm_head rooflines (CUDA events on the decoder's stream)
    vsec, vbytes = sd.profile(0, 20)
    hsec, hbytes = sd.profile(3, 20)
    dsec, dbytes = sd.profile(1, 20)
    step_launches = sd.step_launches()
    L = arch["layers"]
    wall_m, dec_m = reduce(world, [wall, dec], "max")
    # tensor parallel: every rank emits the same tokens
    toks_all = toks if tp else int(reduce(world, [float(toks)], "sum")[0])
    if tp:
        par, scaling = f"tp{world} (target sharded, draft {'sharded' if shard_draft else 'replicated'})", "strong"
    elif split:
        par, scaling = f"dp{world} ({B_all} sequences split over {world} ranks, {B} on rank {rank})", "strong"
    elif world > 1:
        par, scaling = f"replicas x{world} (each rank its own {B} sequences)", "weak"
    else:
        par, scaling = "dp1", "strong"
    peak, peak_kind = peaks()
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", wl["profile"])) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_verify_pass:"):
                    traffic = float(line.split(":")[1])
    except OSError:
        pass
    achieved = vbytes / vsec / 1e9
    res = {
        "metric": METRIC, "value": round(toks_all / dec_m, 3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * wall_m / args.steps, 3), "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "batch": B_all, "K": wl["K"], "prompt": P,
                   "new_tokens": wl["new"], "kv_bits": wl["kv_bits"], "weights": "4-bit g64",
                   "context": ctx + P,
                   "draft": wl["draft"] or f"target's first {wl['draft_layers']} layers",
                   "temperature": wl["temperature"], "top_p": wl["top_p"],
                   "parallelism": par,
                   "l2": f"weights ({vbytes / 1e6:.0f} MB per verify pass) exceed L2; no flush"},
        "e2e": {"value": round(toks_all / wall_m, 3), "unit": "tokens/s",
                "h2d_bytes_per_step": B * P * 4, "d2h_bytes_per_step": B * wl["new"] * 4 + 40},
        "roofline": {"bound": "hbm", "kernel": f"verify pass ({L} layers + lm_head, M={B * (wl['K'] + 1)}"
                                               + (f", per rank of tp{world})" if tp and world > 1 else ")"),
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "frac_of_8000": round(achieved / 8000.0, 4),
                     "algorithmic_bytes": vbytes, "verify_pass_us": round(vsec * 1e6, 2),
                     "traffic": traffic},
        f"lm_head_m{B}": {"us": round(hsec * 1e6, 2), "GBs": round(hbytes / hsec / 1e9, 1)},
        # one draft token (draft forward over B rows incl. its lm_head) and the
        # split of one speculative step (decode time / graph replays): verify
        # pass + K draft tokens + the rest (sampling, acceptance, bookkeeping);
        # verify pass and draft token are timed as CUDA-graph replays, as the
        # decode runs them
        "draft_token": {"us": round(dsec * 1e6, 2), "GBs": round(dbytes / dsec / 1e9, 1),
                        "frac": round(dbytes / dsec / 1e9 / peak, 4), "bytes": dbytes},
        "step": {"ms": round(1e3 * dec / max(1, replays), 3), "verify_ms": round(1e3 * vsec, 3),
                 "draft_ms": round(1e3 * wl["K"] * dsec, 3),
                 "other_ms": round(1e3 * (dec / max(1, replays) - vsec - wl["K"] * dsec), 3),
                 "launches": int(step_launches)},
        "acceptance": {"accepted": acc, "proposed": prop,
                       "rate": round(acc / prop, 4) if prop else None,
                       "tokens_per_step": round(toks / max(1, steps), 3)},
        "clocks": ck, "gpu_launches": int(gpu_launches),
        "sdpa_tc_min_cache": int(lmx.lib().lmx_sdpa_tc_min_cache()),
        "gemm_tcs_max_m": int(lmx.lib().lmx_gemm_tcs_max_m()),
    }
    if world == 1 and rank == 0 and not args.no_cpu and tp:
        tps = toks / max(1, steps)
        r = cpu_sample_composed(wl, arch, darch, args.seed, 2, tps)
        res["cpu_baseline"] = {"value": round(r["value"], 4), "unit": "tokens/s", "cores": r["cores"],
                               "kind": "port", "sample": cpu_composed_sample_text(wl, arch, r, tps)}
    elif world == 1 and rank == 0 and not args.no_cpu:
        r = cpu_sample(wl, prompts, arch, darch, args.seed, args.cpu_steps, 1)
        res["cpu_baseline"] = {"value": round(r["value"], 3), "unit": "tokens/s", "cores": r["cores"],
                               "kind": "port",
                               "sample": cpu_sample_text(r, args.cpu_steps)}
    if rank == 0:
        print(json.dumps(res), flush=True)
    sd.close()
    if draft is not None:
        draft.close()
    target.close()
    if comm is not None:
        barrier(world)
        comm.close()
    return 0


QMM_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
QMM_MS = [1, 2, 4, 5, 8, 12, 16, 32]


def qmm_path(lmx, M):
    """Which K1 kernel takes M rows under the library's current thresholds."""
    mma, tcg = lmx.lib().lmx_mma_min_m(), lmx.lib().lmx_gemv_tc_min_m()
    if mma > 0 and M >= mma and M <= min(64, lmx.lib().lmx_gemm_tcs_max_m()):
        return "mma.sync gemm"
    if mma > 0 and M >= mma:
        return "tcgen05"
    if mma > 0 and tcg > 0 and tcg <= M <= 16:
        return "mma.sync"
    return "gemv"


def qmm_time(lmx, N, K, M, bits, seed=2026):
    """Device time of one quantized matmul launch (BASELINE configs[1] data:
    uniform random codes, scales |N(0,0.02)|/7.5, biases -8 scale): R launches
    over R weight copies (together > 2x L2) captured in one CUDA graph."""
    import torch
    torch.cuda.init()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    KW = K * bits // 32
    wbytes = N * K * bits // 8
    R = max(2, min(64, (320 << 20) // wbytes))
    ws = [torch.randint(-2**31, 2**31 - 1, (N, KW), dtype=torch.int32, device="cuda", generator=gen)
          for _ in range(R)]
    sc = (torch.randn(N, K // 64, device="cuda", generator=gen).abs() * (0.02 / 7.5)).to(torch.bfloat16)
    bi = (-8 * sc.float()).to(torch.bfloat16)
    x = torch.randn(M, K, device="cuda", generator=gen).to(torch.bfloat16)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    st = torch.cuda.Stream()
    S = C.c_void_p(st.cuda_stream)

    def run():
        for w in ws:
            lmx.call("lmx_quantized_matmul", x.data_ptr(), w.data_ptr(), sc.data_ptr(), bi.data_ptr(),
                     y.data_ptr(), M, N, K, 64, bits, S)

    with torch.cuda.stream(st):
        run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        run()
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e-3 / R)
    t = statistics.median(ts)
    del g
    byts = wbytes + N * (K // 64) * 4 + M * K * 2 + M * N * 2
    return dict(N=N, K=K, M=M, bits=bits, us=round(t * 1e6, 2), GBs=round(byts / t / 1e9, 1),
                path=qmm_path(lmx, M))


def sdpa_path(lmx, rows, cap):
    """Which K2 kernel runs for `rows` query rows per KV head over a cache of
    `cap` rows under the library's current thresholds."""
    mma, long_cache = lmx.lib().lmx_mma_min_m(), lmx.lib().lmx_sdpa_tc_min_cache()
    return "tensor-core" if mma > 0 and (rows >= mma or (long_cache > 0 and cap >= long_cache)) else "cuda-core"


def sdpa_time(lmx, B, T, Hq, Hk, cap, bits, seed=2026):
    """Device time of one lmx_sdpa_decode launch over an affine (4/8-bit) or
    bf16 cache with every sequence at length cap - T (uniform random codes,
    scales |N(0,0.2)|/(2^bits-1), biases N(0,1)): R launches over R cache
    copies (together > 2x L2) captured in one CUDA graph."""
    import torch
    torch.cuda.init()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    D = 128
    rows = B * Hk * cap
    row_bytes = D * 2 if bits == 16 else D * bits // 8 + 8
    cbytes = 2 * rows * row_bytes
    R = max(1, min(16, (320 << 20) // cbytes))
    keep, descs = [], []
    lens = torch.full((B,), cap - T, dtype=torch.int32, device="cuda")
    for _ in range(R):
        d = lmx.KvDesc(batch=B, kv_heads=Hk, head_dim=D, capacity=cap, bits=bits, lengths=lens.data_ptr())
        if bits == 16:
            k = torch.randn(rows * D, device="cuda", generator=gen).to(torch.bfloat16)
            v = torch.randn(rows * D, device="cuda", generator=gen).to(torch.bfloat16)
            d.k, d.v = k.data_ptr(), v.data_ptr()
            keep += [k, v]
        else:
            t = [torch.randint(-2**31, 2**31 - 1, (rows * D * bits // 32,), dtype=torch.int32, device="cuda",
                               generator=gen) for _ in range(2)]
            sc = [(torch.randn(rows * 2, device="cuda", generator=gen).abs() * (0.2 / (2**bits - 1)))
                  .to(torch.bfloat16) for _ in range(2)]
            bi = [torch.randn(rows * 2, device="cuda", generator=gen).to(torch.bfloat16) for _ in range(2)]
            d.k_packed, d.v_packed = t[0].data_ptr(), t[1].data_ptr()
            d.k_scales, d.v_scales = sc[0].data_ptr(), sc[1].data_ptr()
            d.k_biases, d.v_biases = bi[0].data_ptr(), bi[1].data_ptr()
            keep += t + sc + bi
        descs.append(d)
    q = torch.randn(B * T * Hq * D, device="cuda", generator=gen).to(torch.bfloat16)
    out = torch.empty_like(q)
    nbytes = lmx.lib().lmx_sdpa_scratch_bytes(B, T, Hq, Hk, cap)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    st = torch.cuda.Stream()
    S = C.c_void_p(st.cuda_stream)
    scale = float(np.float32(1.0 / np.sqrt(D)))

    def run():
        for d in descs:
            lmx.call("lmx_sdpa_decode", q.data_ptr(), C.byref(d), T, Hq, scale, scratch.data_ptr(), nbytes,
                     out.data_ptr(), S)

    with torch.cuda.stream(st):
        run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        run()
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e-3 / R)
    t = statistics.median(ts)
    del g
    byts = 2 * B * Hk * cap * row_bytes + 2 * B * T * Hq * D * 2  # every row is visible (lengths cap - T)
    G = Hq // Hk
    return dict(B=B, T=T, Hq=Hq, Hk=Hk, cap=cap, bits=bits, us=round(t * 1e6, 2), GBs=round(byts / t / 1e9, 1),
                path=sdpa_path(lmx, G * T, cap))


def _graph_time(run, reps=5):
    """Median device time of one replay of run() captured in a CUDA graph."""
    import torch
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        run(st)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        run(st)
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e-3)
    del g
    return statistics.median(ts)


def moe_time(lmx, M, H, I, E, k, bits, seed=2026):
    """Device time of lmx_moe_experts (configuration 4's routed experts):
    E experts of uniform random codes, top-k expert ids drawn per token; R
    expert sets (together > 2x L2) rotated inside one graph.  Algorithmic
    bytes = the unique experts touched x (gate + up + down packed weights and
    scales / biases) + activations."""
    import torch
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    rng = np.random.RandomState(seed)
    per_expert = 3 * I * H * bits // 8 + 3 * I * (H // 64) * 4
    R = max(1, min(8, (320 << 20) // (E * per_expert)))

    def qw(N, K):
        w = torch.randint(-2**31, 2**31 - 1, (E, N, K * bits // 32), dtype=torch.int32, device="cuda", generator=gen)
        s = (torch.rand(E, N, K // 64, device="cuda", generator=gen) * 0.01 + 0.002).to(torch.bfloat16)
        b = (-torch.rand(E, N, K // 64, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
        return (w, s, b), lmx.QWeights(w=w.data_ptr(), scales=s.data_ptr(), biases=b.data_ptr())

    sets = [[qw(I, H), qw(I, H), qw(H, I)] for _ in range(R)]
    idx_np = np.stack([rng.choice(E, k, replace=False) for _ in range(M)]).astype(np.int32)
    idx = torch.from_numpy(idx_np).cuda()
    w = torch.full((M, k), 1.0 / k, dtype=torch.float32, device="cuda")
    x = torch.randn(M, H, device="cuda", generator=gen).to(torch.bfloat16)
    act = torch.empty(M, k, I, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")

    def run(st):
        for g3 in sets:
            lmx.call("lmx_moe_experts", x.data_ptr(), M, H, I, E, k, idx.data_ptr(), w.data_ptr(), C.byref(g3[0][1]),
                     C.byref(g3[1][1]), C.byref(g3[2][1]), bits, act.data_ptr(), y.data_ptr(),
                     C.c_void_p(st.cuda_stream))

    t = _graph_time(run) / R
    uniq = len(set(idx_np.ravel().tolist()))
    byts = uniq * per_expert + M * H * 2 * 2 + M * k * I * 2 * 2
    return dict(op="moe_experts", M=M, H=H, I=I, E=E, k=k, bits=bits, unique_experts=uniq,
                us=round(t * 1e6, 2), GBs=round(byts / t / 1e9, 1), bytes=byts)


def gdn_time(lmx, B, T, Hk, Hv, seed=2026):
    """Device time of lmx_gdn_verify + lmx_gdn_commit (configuration 4's
    Gated DeltaNet layer core).  Algorithmic bytes = fp32 state read + T
    snapshots written + the state rewritten by the commit + inputs / output."""
    import torch
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    D = 128
    CD = 2 * Hk * D + Hv * D
    bf = lambda *s: (torch.randn(*s, device="cuda", generator=gen)).to(torch.bfloat16)
    t_ = dict(qkv=bf(B, T, CD), z=bf(B, T, Hv * D), b=bf(B, T, Hv), a=bf(B, T, Hv), conv_w=bf(CD, 4) * 0.5,
              a_log=torch.zeros(Hv, device="cuda"), dt_bias=bf(Hv), norm_w=torch.ones(D, dtype=torch.bfloat16,
                                                                                      device="cuda"),
              conv_state=bf(B, 3, CD), state=torch.randn(B, Hv, D, D, device="cuda", generator=gen) * 0.05,
              snap=torch.empty(B, T, Hv, D, D, device="cuda"), out=torch.empty(B, T, Hv * D, dtype=torch.bfloat16,
                                                                              device="cuda"))
    t_["scratch"] = torch.empty(lmx.lib().lmx_gdn_scratch_bytes(B, T, Hk, Hv), dtype=torch.uint8, device="cuda")
    g = lmx.GdnDesc(batch=B, T=T, k_heads=Hk, v_heads=Hv, eps=1e-6)
    for f, k in (("qkv", "qkv"), ("z", "z"), ("b", "b"), ("a", "a"), ("conv_w", "conv_w"), ("a_log", "a_log"),
                 ("dt_bias", "dt_bias"), ("norm_w", "norm_w"), ("conv_state", "conv_state"), ("state", "state"),
                 ("state_snap", "snap"), ("out", "out"), ("scratch", "scratch")):
        setattr(g, f, t_[k].data_ptr())
    acc = torch.full((B,), T - 1, dtype=torch.int32, device="cuda")

    def run(st):
        s = C.c_void_p(st.cuda_stream)
        lmx.call("lmx_gdn_verify", C.byref(g), s)
        lmx.call("lmx_gdn_commit", C.byref(g), acc.data_ptr(), s)

    t = _graph_time(run)
    st_bytes = B * Hv * D * D * 4
    byts = st_bytes * (2 + T) + B * T * (CD + 2 * Hv * D) * 2 + B * 3 * CD * 2 * 2
    return dict(op="gdn_verify+commit", B=B, T=T, Hk=Hk, Hv=Hv, us=round(t * 1e6, 2),
                GBs=round(byts / t / 1e9, 1), bytes=byts)


def run_qmm(args):
    lmx = _load("lmx", os.path.join(ROOT, "lemon-mlx-engine_b200", "lmx.py"))
    lmx.call("lmx_set_device", 0)
    if args.gemm_tcs_max_m >= 0:
        lmx.call("lmx_set_gemm_tcs_max_m", args.gemm_tcs_max_m)
    peak, kind = peaks()
    if args.qmm:
        N, K, M, bits = [int(v) for v in args.qmm.split(",")]
        rows = [qmm_time(lmx, N, K, M, bits)]
    else:
        rows = [qmm_time(lmx, N, K, M, bits) for bits in (4, 8) for N, K in QMM_SHAPES for M in QMM_MS]
    best = max(r["GBs"] for r in rows)
    print(json.dumps({"metric": "quantized_matmul GB/s (BASELINE configs[1] sweep)", "value": best,
                      "unit": "GB/s", "n_gpus": 1, "higher_is_better": True, "data": "synthetic",
                      "peak": peak, "peak_source": kind, "l2": "weight copies > 2x L2 per graph",
                      "sweep": rows}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed generations (default: the workload's, about a minute of decode)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="lmx", choices=["lmx", "reference"])
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--seed", type=int, default=2026)
    ap.add_argument("--cpu-steps", type=int, default=None,
                    help="speculative steps in the CPU sample (default: 6, or the workload's own)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1 without tensor parallelism: every rank decodes the workload's whole batch "
                         "(weak scaling) instead of its share of one batch")
    ap.add_argument("--profile-verify", type=int, default=0,
                    help="only prefill the workload and run N verify passes inside the NVTX "
                         "range lmx_verify_pass (for ncu --nvtx-include)")
    ap.add_argument("--profile-draft", type=int, default=0,
                    help="only prefill the workload and run N single-token draft forwards inside the "
                         "NVTX range lmx_draft_token (for ncu --nvtx-include)")
    ap.add_argument("--layers", type=int, default=0,
                    help="with --profile-verify / --profile-draft only: build the target with this many "
                         "layers (same per-layer shapes; a small case for ncu captures)")
    ap.add_argument("--qmm-sweep", action="store_true",
                    help="op-level quantized_matmul sweep (BASELINE configs[1]) instead of decoding")
    ap.add_argument("--qmm", default="", help="one op-level shape N,K,M,bits (e.g. for ncu)")
    ap.add_argument("--moe", default="", help="op-level routed experts M,H,I,E,k,bits (configuration 4: "
                                              "12,2048,512,512,10,4)")
    ap.add_argument("--gdn", default="", help="op-level Gated DeltaNet verify + commit B,T,Hk,Hv (configuration 4: "
                                              "4,3,16,32)")
    ap.add_argument("--replicated-draft", action="store_true",
                    help="tensor parallel: a whole copy of the draft on every rank instead of its shard")
    ap.add_argument("--gemm-tcs-max-m", type=int, default=-1,
                    help="set lmx_set_gemm_tcs_max_m first: M up to this bound on the mid-batch mma.sync GEMM "
                         "(0: tcgen05 for every M at or above the threshold)")
    ap.add_argument("--sdpa-tc-min-cache", type=int, default=-1,
                    help="set lmx_set_sdpa_tc_min_cache first (0: by row count only; a large value keeps "
                         "single-token decode attention on the canonical kernel)")
    ap.add_argument("--sdpa", default="", help="one op-level attention shape B,T,Hq,Hk,cap,bits (e.g. "
                                               "16,5,64,8,8300,8 = one Llama-3-70B verify layer)")
    args = ap.parse_args()
    if args.qmm_sweep or args.qmm:
        return run_qmm(args)
    if args.moe or args.gdn:
        lmx = _load("lmx", os.path.join(ROOT, "lemon-mlx-engine_b200", "lmx.py"))
        lmx.call("lmx_set_device", 0)
        if args.moe:
            M, H_, I, E, k, bits = [int(v) for v in args.moe.split(",")]
            print(json.dumps(moe_time(lmx, M, H_, I, E, k, bits)), flush=True)
        if args.gdn:
            B, T, Hk, Hv = [int(v) for v in args.gdn.split(",")]
            print(json.dumps(gdn_time(lmx, B, T, Hk, Hv)), flush=True)
        return 0
    if args.sdpa:
        lmx = _load("lmx", os.path.join(ROOT, "lemon-mlx-engine_b200", "lmx.py"))
        lmx.call("lmx_set_device", 0)
        if args.sdpa_tc_min_cache >= 0:
            lmx.call("lmx_set_sdpa_tc_min_cache", args.sdpa_tc_min_cache)
        B, T, Hq, Hk, cap, bits = [int(v) for v in args.sdpa.split(",")]
        print(json.dumps(sdpa_time(lmx, B, T, Hq, Hk, cap, bits)), flush=True)
        return 0
    wl = WORKLOADS[args.workload]
    if args.layers and not (args.profile_verify or args.profile_draft):
        ap.error("--layers is only for the profiling runs")
    if args.steps is None:
        args.steps = wl.get("steps", 10)
    if args.cpu_steps is None:
        args.cpu_steps = wl.get("cpu_steps", 6)
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            return run_reference(args, wl, world, rank)
        if wl.get("hybrid"):
            return run_hybrid(args, wl, world, rank, local)
        return run_lmx(args, wl, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
