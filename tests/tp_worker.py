"""One rank of a tensor-parallel run, launched by test_tp_gpu.py through
torch.distributed.run (one process per GPU, handles exchanged over gloo).

Every rank builds its shard of the same seeded models and runs
  * forwards through a cache with a synthetic context (logits of this rank's
    vocabulary slice, gathered to rank 0 and concatenated), once per
    tensor-core threshold, and
  * a greedy speculative session: Llama-style target (tensor-parallel) with a
    replicated draft, 8-bit KV, a synthetic context before the prompt, and
    the same session with the draft sharded over the communicator too;
  * with --ckpt, forwards of a checkpoint loaded as tensor-parallel shards;
and rank 0 writes everything to --out (.npz) for the parent to compare with
the oracle's tensor-parallel emulation.  Every rank must produce the same
stream; the worker checks that itself.
"""
import argparse
import ctypes as C
import datetime
import importlib.util
import os

import numpy as np
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

TARGET = dict(hidden=512, layers=2, inter=1024, heads=8, kv_heads=2, head_dim=128, vocab=4096,
              rope_theta=5e5, eps=1e-5, qk_norm=0, tied=0, bits=4, group_size=64)
TARGET_TIED8 = dict(TARGET, tied=1, bits=8)
DRAFT = dict(TARGET, layers=1, tied=1)
SEED = 2024
CTX, CTX_SEED = 60, 5
B, P, K, MT = 3, 16, 4, 40
FWD_BLOCKS = (8, 5, 1)


def load_lmx():
    spec = importlib.util.spec_from_file_location("lmx", os.path.join(ROOT, "lemon-mlx-engine_b200", "lmx.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def prompts():
    return np.random.RandomState(9).randint(0, TARGET["vocab"], (B, P)).astype(np.int32)


def forward_tokens():
    rng = np.random.RandomState(17)
    return [rng.randint(0, TARGET["vocab"], (B, T)).astype(np.int32) for T in FWD_BLOCKS]


def gather_concat(x, axis):
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, x)
    return np.concatenate(parts, axis=axis)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--ckpt", default="", help="checkpoint directory to load as tp shards")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    lmx = load_lmx()
    lmx.call("lmx_set_device", local)
    comm = lmx.TpComm.from_process_group(max_rows=B * 32, max_hidden=TARGET["hidden"])
    res = {}

    # forwards over a synthetic context, exact mode (0) and tensor-core mode (16)
    m = lmx.Model(TARGET_TIED8, SEED, comm=comm)
    vl = TARGET["vocab"] // world
    for mma in (0, 16):
        lmx.call("lmx_set_mma_min_m", mma)
        gc = C.c_void_p()
        lmx.call("lmx_cache_create", m.h, TARGET["layers"], B, 128, 8, 8, C.byref(gc))
        lmx.call("lmx_cache_fill_synthetic", gc, CTX, CTX_SEED, 0x40000000)
        for i, tok in enumerate(forward_tokens()):
            T = tok.shape[1]
            lg = np.zeros((B, T, vl), np.uint16)
            lmx.call("lmx_forward", m.h, gc, TARGET["layers"], tok.ctypes.data, B, T, lg.ctypes.data)
            res[f"logits_mma{mma}_{i}"] = gather_concat(lg, 2)
        lmx.call("lmx_cache_free", gc)
    m.close()

    # a mixed-precision checkpoint loaded as this rank's shard, exact mode
    if args.ckpt:
        lmx.call("lmx_set_mma_min_m", 0)
        m = lmx.Model.load(args.ckpt, comm=comm)
        c = m.cfg
        gc = C.c_void_p()
        lmx.call("lmx_cache_create", m.h, c["layers"], B, 128, 16, 8, C.byref(gc))
        for i, tok in enumerate(forward_tokens()):
            T = tok.shape[1]
            lg = np.zeros((B, T, c["vocab"] // world), np.uint16)
            lmx.call("lmx_forward", m.h, gc, c["layers"], tok.ctypes.data, B, T, lg.ctypes.data)
            res[f"ckpt_logits_{i}"] = gather_concat(lg, 2)
        lmx.call("lmx_cache_free", gc)
        m.close()

    # greedy speculative session, exact mode
    lmx.call("lmx_set_mma_min_m", 0)
    tm = lmx.Model(TARGET, SEED, comm=comm)
    dm = lmx.Model(DRAFT, SEED + 1)
    sd = lmx.SpecDecoder(tm, dm, 1, B, K, MT, P, kv_bits=8, context_len=CTX, context_seed=CTX_SEED)
    sd.prefill(prompts())
    sd.decode()
    out, stats = sd.result()
    sd.close()
    tm.close()
    dm.close()
    streams = [None] * world
    dist.all_gather_object(streams, out)
    for r in range(1, world):
        if not np.array_equal(streams[r], streams[0]):
            raise SystemExit(f"rank {r} emitted a different stream than rank 0")
    res["stream"] = out
    res["accepted"] = np.array(stats["accepted"])

    # the same session with the draft sharded over the communicator too
    tm = lmx.Model(TARGET, SEED, comm=comm)
    dm = lmx.Model(DRAFT, SEED + 1, comm=comm)
    sd = lmx.SpecDecoder(tm, dm, 1, B, K, MT, P, kv_bits=8, context_len=CTX, context_seed=CTX_SEED)
    sd.prefill(prompts())
    sd.decode()
    out, stats = sd.result()
    sd.close()
    tm.close()
    dm.close()
    dist.all_gather_object(streams, out)
    for r in range(1, world):
        if not np.array_equal(streams[r], streams[0]):
            raise SystemExit(f"rank {r} emitted a different stream than rank 0 (tp draft)")
    res["stream_tp_draft"] = out
    res["accepted_tp_draft"] = np.array(stats["accepted"])
    dist.barrier()
    comm.close()
    if rank == 0:
        np.savez(args.out, **res)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
