"""Generate golden vectors from the reference's own Python functions.

Run where the reference tree is mounted; its root directory is the required
--ref argument.  It imports

  debug_numerical_trace.py : dequantize_4bit_affine, rms_norm, quantized_matmul_4bit
  debug_layer0_reference.py: dequantize_weight (4- and 8-bit)

which pin the MLX affine packing order (LSB-first) and w = q*scale + bias, and
stores their outputs on small seeded inputs in golden.npz.  The fixtures are
committed; the tests read only the .npz, never the reference tree.
"""
import argparse
import importlib.util
import os
import sys

import numpy as np


def load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # both files guard main() behind __name__
    return mod


def bf16_round(f32):
    u = np.asarray(f32, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root directory of the reference tree")
    ap.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "golden.npz"))
    a = ap.parse_args()
    trace = load(os.path.join(a.ref, "debug_numerical_trace.py"), "ref_trace")
    layer0 = load(os.path.join(a.ref, "debug_layer0_reference.py"), "ref_layer0")

    rng = np.random.RandomState(20261201)
    out = {}
    # 4-bit: packed words, bf16 scales/biases (as bit patterns), activations.
    N, K = 24, 256
    w4 = rng.randint(0, 2**32, size=(N, K // 8), dtype=np.uint64).astype(np.uint32)
    s4 = bf16_round(np.abs(rng.normal(0, 0.02, (N, K // 64))).astype(np.float32) / 7.5)
    b4 = bf16_round(-8.0 * (s4.astype(np.uint32) << 16).view(np.float32))
    x4 = bf16_round(rng.normal(0, 1, (3, K)).astype(np.float32))
    sf = (s4.astype(np.uint32) << 16).view(np.float32)
    bf = (b4.astype(np.uint32) << 16).view(np.float32)
    xf = (x4.astype(np.uint32) << 16).view(np.float32)
    out.update(q4_w=w4, q4_s=s4, q4_b=b4, q4_x=x4)
    # unit scale / zero bias -> the dequantized values are the raw codes
    out["q4_codes"] = trace.dequantize_4bit_affine(w4, np.ones_like(sf), np.zeros_like(bf))
    out["q4_deq"] = trace.dequantize_4bit_affine(w4, sf, bf)
    out["q4_deq_l0"] = layer0.dequantize_weight(w4, sf, bf, group_size=64, bits=4)
    out["q4_qmm"] = trace.quantized_matmul_4bit(xf, w4, sf, bf)
    # 8-bit through the generic reference dequantizer
    w8 = rng.randint(0, 2**32, size=(N, K // 4), dtype=np.uint64).astype(np.uint32)
    s8 = bf16_round(np.abs(rng.normal(0, 0.02, (N, K // 64))).astype(np.float32) / 127.5)
    b8 = bf16_round(-128.0 * (s8.astype(np.uint32) << 16).view(np.float32))
    s8f = (s8.astype(np.uint32) << 16).view(np.float32)
    b8f = (b8.astype(np.uint32) << 16).view(np.float32)
    out.update(q8_w=w8, q8_s=s8, q8_b=b8)
    out["q8_codes"] = layer0.dequantize_weight(w8, np.ones_like(s8f), np.zeros_like(b8f), 64, 8)
    out["q8_deq"] = layer0.dequantize_weight(w8, s8f, b8f, 64, 8)
    out["q8_qmm"] = xf @ out["q8_deq"].T
    # rms_norm
    xr = bf16_round(rng.normal(0, 1.5, (4, 1024)).astype(np.float32))
    wr = bf16_round(rng.normal(1, 0.1, (1024,)).astype(np.float32))
    out.update(rms_x=xr, rms_w=wr)
    out["rms_y"] = trace.rms_norm((xr.astype(np.uint32) << 16).view(np.float32),
                                  (wr.astype(np.uint32) << 16).view(np.float32), eps=1e-6)
    np.savez_compressed(a.out, **out)
    print("wrote", a.out, sorted(out))


if __name__ == "__main__":
    sys.exit(main())
