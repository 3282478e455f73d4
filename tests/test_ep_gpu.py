"""Expert parallelism for configuration 4 on 2 GPUs (one process per GPU):
each rank holds half of every MoE block's experts; the routed experts' slot
outputs are exchanged over NVLink and combined in slot order.  Exact mode:
the trunk's logits and the MTP speculative stream are bit-identical to the
single-GPU model's (and hence to the oracle, test_hybrid_model_gpu)."""
import ctypes as C
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import ep_worker as W
import hybrid_cases as H

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_ep2_bit_identical_to_one_gpu(lmx, cuda, mma_threshold, tmp_path):
    if cuda.cuda.device_count() < 2:
        pytest.skip("expert-parallel test needs 2 GPUs")
    out = str(tmp_path / "ep2.npz")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", os.path.join(HERE, "ep_worker.py"),
           "--out", out]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, f"ep worker failed:\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    ep = dict(np.load(out))
    mma_threshold(0)
    h = C.c_void_p()
    lmx.call("lmx_hybrid_create", C.byref(lmx.HybridConfig(**H.TINY_HYBRID)), W.SEED, C.byref(h))
    try:
        logits, stream = W.run(lmx, h, H.TINY_HYBRID)
    finally:
        lmx.lib().lmx_hybrid_free(h)
    for i, lg in enumerate(logits):
        np.testing.assert_array_equal(ep[f"logits{i}"], lg)
    np.testing.assert_array_equal(ep["stream"], stream)
