"""One rank of an expert-parallel run of configuration 4's hybrid model,
launched by test_ep_gpu.py through torch.distributed.run (one process per
GPU, handles exchanged over gloo).  Every rank builds its shard of the
experts of the same seeded model and runs, in exact mode, the trunk's
logits over prefill and decode blocks and an MTP speculative stream; rank 0
writes them to --out (.npz).  Every rank must produce the same results (the
worker checks that itself)."""
import argparse
import ctypes as C
import datetime
import importlib.util
import os
import sys

import numpy as np
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import hybrid_cases as H  # noqa: E402

SEED = 77
B, P, MT, CAP = 3, 20, 24, 96
BLOCK_T = (37, 5, 1, 3)


def load_lmx():
    spec = importlib.util.spec_from_file_location("lmx", os.path.join(ROOT, "lemon-mlx-engine_b200", "lmx.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def blocks(V):
    rng = np.random.RandomState(3)
    return [rng.randint(0, V, (B, T)).astype(np.int32) for T in BLOCK_T]


def prompts(V):
    return np.random.RandomState(5).randint(0, V, (B, P)).astype(np.int32)


def run(lmx, h, cfg):
    """Logits of every block and the MTP stream through model h."""
    V = cfg["vocab"]
    st = C.c_void_p()
    lmx.call("lmx_hybrid_state_create", h, B, CAP, 16, 40, C.byref(st))
    logits = []
    for tok in blocks(V):
        T = tok.shape[1]
        lg = np.zeros((B, T, V), np.uint16)
        lmx.call("lmx_hybrid_forward", h, st, tok.ctypes.data, B, T, lg.ctypes.data)
        logits.append(lg)
    lmx.lib().lmx_hybrid_state_free(st)
    sp = C.c_void_p()
    lmx.call("lmx_hybrid_spec_create", h, B, MT, P, 16, C.byref(sp))
    p = prompts(V)
    lmx.call("lmx_hybrid_spec_prefill", sp, p.ctypes.data)
    sec = C.c_double()
    lmx.call("lmx_hybrid_spec_decode", sp, 1, C.byref(sec))
    out = np.zeros((B, MT), np.int32)
    stats = np.zeros(5, np.int64)
    lmx.call("lmx_hybrid_spec_result", sp, out.ctypes.data, stats.ctypes.data)
    lmx.lib().lmx_hybrid_spec_free(sp)
    return logits, out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    lmx = load_lmx()
    lmx.call("lmx_set_device", local)
    lmx.call("lmx_set_mma_min_m", 0)
    cfg = H.TINY_HYBRID
    comm = lmx.TpComm.from_process_group(max_rows=B * 40 * cfg["top_k"], max_hidden=cfg["hidden"])
    h = C.c_void_p()
    lmx.call("lmx_hybrid_create_ep", C.byref(lmx.HybridConfig(**cfg)), SEED, comm.h, C.byref(h))
    logits, out = run(lmx, h, cfg)
    code = C.c_uint(0)
    lmx.call("lmx_device_error", C.byref(code), 1)
    assert code.value == 0, hex(code.value)
    streams = [None] * dist.get_world_size()
    dist.all_gather_object(streams, out)
    for s in streams:
        np.testing.assert_array_equal(s, out)
    dist.barrier()
    lmx.lib().lmx_hybrid_free(h)
    comm.close()
    if rank == 0:
        np.savez(args.out, stream=out, **{f"logits{i}": x for i, x in enumerate(logits)})
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
