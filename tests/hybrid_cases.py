"""Seeded inputs for the hybrid-model ops (Gated DeltaNet verify step, MoE
router and experts) and float64 NumPy restatements of the reference math,
shared by the CPU tests (oracle vs the formulas) and the GPU tests (device vs
oracle).  Reference formulas: Qwen3NextGatedDeltaNet (src/llm/models/
qwen3_next.cpp:216-403), gated_delta.cpp:603-650, 885-921, 948-999;
Qwen3NextSparseMoeBlock (qwen3_next.cpp:452-490), SwitchGLU
(src/common/switch_layers.cpp:200-245)."""
import ctypes as C

import numpy as np

import oracle_lib as O

D = 128


def bf16(a):
    return O.f32_to_bf16(np.asarray(a, np.float32))


def gdn_case(seed, B, T, Hk, Hv, state_scale=0.05):
    rng = np.random.RandomState(seed)
    CD = 2 * Hk * D + Hv * D
    c = dict(B=B, T=T, Hk=Hk, Hv=Hv, eps=1e-6)
    c["qkv"] = bf16(rng.normal(0, 1, (B, T, CD)))
    c["z"] = bf16(rng.normal(0, 1, (B, T, Hv * D)))
    c["b"] = bf16(rng.normal(0, 1, (B, T, Hv)))
    c["a"] = bf16(rng.normal(0, 1, (B, T, Hv)))
    c["conv_w"] = bf16(rng.normal(0, 0.5, (CD, 4)))
    c["a_log"] = rng.uniform(-1.0, 1.0, Hv).astype(np.float32)
    c["dt_bias"] = bf16(rng.normal(0, 0.5, Hv))
    c["norm_w"] = bf16(rng.uniform(0.5, 1.5, D))
    c["conv_state"] = bf16(rng.normal(0, 1, (B, 3, CD)))
    c["state"] = (rng.normal(0, state_scale, (B, Hv, D, D))).astype(np.float32)
    return c


def oracle_gdn(c):
    B, T, Hk, Hv = c["B"], c["T"], c["Hk"], c["Hv"]
    snap = np.zeros((B, T, Hv, D, D), np.float32)
    out = np.zeros((B, T, Hv * D), np.uint16)
    rc = O.lib().orc_gdn_verify(B, T, Hk, Hv, O.ptr(c["qkv"]), O.ptr(c["z"]), O.ptr(c["b"]), O.ptr(c["a"]),
                                O.ptr(c["conv_w"]), O.ptr(c["a_log"]), O.ptr(c["dt_bias"]), O.ptr(c["norm_w"]),
                                c["eps"], O.ptr(c["conv_state"]), O.ptr(c["state"]), O.ptr(snap), O.ptr(out))
    assert rc == 0
    return out, snap


def oracle_commit(c, snap, acc):
    B, T, Hk, Hv = c["B"], c["T"], c["Hk"], c["Hv"]
    state = c["state"].copy()
    conv = c["conv_state"].copy()
    acc = np.ascontiguousarray(acc, np.int32)
    assert O.lib().orc_gdn_commit(B, T, Hk, Hv, O.ptr(c["qkv"]), O.ptr(snap), O.ptr(acc), O.ptr(state),
                                  O.ptr(conv)) == 0
    return state, conv


def reference_gdn(c):
    """float64 restatement of the reference step (no intermediate rounding)."""
    B, T, Hk, Hv = c["B"], c["T"], c["Hk"], c["Hv"]
    f = lambda u: O.bf16_to_f32(u).astype(np.float64)
    qkv, z, bb, aa = f(c["qkv"]), f(c["z"]), f(c["b"]), f(c["a"])
    w, dtb, nw = f(c["conv_w"]), f(c["dt_bias"]), f(c["norm_w"])
    win = np.concatenate([f(c["conv_state"]), qkv], 1)  # [B, 3+T, CD]
    sig = lambda x: 1.0 / (1.0 + np.exp(-x))
    S = c["state"].astype(np.float64).copy()
    out = np.zeros((B, T, Hv, D))
    rep = Hv // Hk
    for t in range(T):
        y = (win[:, t:t + 4, :] * w.T[None]).sum(1)
        y = y * sig(y)
        q = y[:, :Hk * D].reshape(B, Hk, D)
        k = y[:, Hk * D:2 * Hk * D].reshape(B, Hk, D)
        v = y[:, 2 * Hk * D:].reshape(B, Hv, D)
        rms = lambda x: x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6)
        q = rms(q) / D
        k = rms(k) / np.sqrt(D)
        q, k = np.repeat(q, rep, 1), np.repeat(k, rep, 1)
        beta = sig(bb[:, t])
        g = np.exp(-np.exp(c["a_log"].astype(np.float64))[None] * np.log1p(np.exp(aa[:, t] + dtb[None])))
        S = S * g[:, :, None, None]
        kv = (S * k[:, :, None, :]).sum(-1)
        delta = (v - kv) * beta[:, :, None]
        S = S + delta[:, :, :, None] * k[:, :, None, :]
        yv = (S * q[:, :, None, :]).sum(-1)
        zn = z[:, t].reshape(B, Hv, D)
        normed = yv / np.sqrt((yv * yv).mean(-1, keepdims=True) + c["eps"]) * nw
        out[:, t] = zn * sig(zn) * normed
    return out.reshape(B, T, Hv * D), S


def moe_route_case(seed, rows, E):
    rng = np.random.RandomState(seed)
    l = rng.normal(0, 2, (rows, E)).astype(np.float32)
    l[0, 5] = l[0, 7] = l[0].max() + 1  # a tie at the top: the lower index first
    return bf16(l)


def oracle_route(logits, k):
    rows, E = logits.shape
    idx = np.zeros((rows, k), np.int32)
    w = np.zeros((rows, k), np.float32)
    assert O.lib().orc_moe_route(O.ptr(logits), rows, E, k, O.ptr(idx), O.ptr(w)) == 0
    return idx, w


def moe_experts_case(seed, M, H, I, E, k, bits):
    rng = np.random.RandomState(seed)
    per = 32 // bits

    def qw(N, K):
        w = rng.randint(0, 2**32, (E, N, K // per), dtype=np.uint64).astype(np.uint32)
        s = bf16(rng.uniform(0.002, 0.02, (E, N, K // 64)) / (2**bits - 1) * 15)
        b = bf16(-rng.uniform(0.01, 0.15, (E, N, K // 64)))
        return w, s, b

    c = dict(M=M, H=H, I=I, E=E, k=k, bits=bits)
    c["x"] = bf16(rng.normal(0, 1, (M, H)))
    c["gate"], c["up"], c["down"] = qw(I, H), qw(I, H), qw(H, I)
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(M)]).astype(np.int32)
    idx[M - 1] = idx[0]  # two tokens routed to the same experts
    c["idx"] = idx
    wt = rng.uniform(0.1, 1.0, (M, k)).astype(np.float32)
    c["w"] = (wt / wt.sum(1, keepdims=True)).astype(np.float32)
    return c


def oracle_experts(c):
    y = np.zeros((c["M"], c["H"]), np.uint16)
    g, u, d = c["gate"], c["up"], c["down"]
    assert O.lib().orc_moe_experts(O.ptr(c["x"]), c["M"], c["H"], c["I"], c["E"], c["k"], O.ptr(c["idx"]),
                                   O.ptr(c["w"]), O.ptr(g[0]), O.ptr(g[1]), O.ptr(g[2]), O.ptr(u[0]), O.ptr(u[1]),
                                   O.ptr(u[2]), O.ptr(d[0]), O.ptr(d[1]), O.ptr(d[2]), c["bits"], O.ptr(y)) == 0
    return y


def reference_experts(c):
    """float64: dequantize (w = q*s + b) and multiply; swiglu; weighted sum."""
    bits = c["bits"]

    def deq(qw3, e):
        w, s, b = qw3
        N = w.shape[1]
        K = w.shape[2] * 32 // bits
        codes = np.zeros((N, K), np.float64)
        for j in range(32 // bits):
            codes[:, j::32 // bits] = (w[e] >> np.uint32(j * bits)) & np.uint32(2**bits - 1)
        sc = np.repeat(O.bf16_to_f32(s[e]).astype(np.float64), 64, 1)
        bi = np.repeat(O.bf16_to_f32(b[e]).astype(np.float64), 64, 1)
        return codes * sc + bi

    x = O.bf16_to_f32(c["x"]).astype(np.float64)
    y = np.zeros((c["M"], c["H"]))
    for m in range(c["M"]):
        for j in range(c["k"]):
            e = c["idx"][m, j]
            g = deq(c["gate"], e) @ x[m]
            u = deq(c["up"], e) @ x[m]
            a = g / (1 + np.exp(-g)) * u
            y[m] += c["w"][m, j] * (deq(c["down"], e) @ a)
    return y


TINY_HYBRID = dict(hidden=512, layers=4, attn_every=2, heads=4, kv_heads=2, lin_k_heads=2, lin_v_heads=4,
                   experts=8, top_k=2, expert_inter=512, shared_inter=512, vocab=1000, rope_theta=1e7, eps=1e-6,
                   bits=4)


def oracle_hybrid(cfg, seed):
    return O.lib().orc_hybrid_create(C.byref(O.HybridCfg(**cfg)), seed)


def oracle_hybrid_forward_blocks(o, cfg, B, cap, kv_bits, blocks):
    st = O.lib().orc_hybrid_state_create(o, B, cap, kv_bits)
    outs = []
    for tok in blocks:
        T = tok.shape[1]
        lg = np.zeros((B, T, cfg["vocab"]), np.uint16)
        assert O.lib().orc_hybrid_forward(o, st, O.ptr(np.ascontiguousarray(tok)), B, T, O.ptr(lg)) == 0
        outs.append(lg)
    O.lib().orc_hybrid_state_free(st)
    return outs


def oracle_hybrid_spec(o, prompts, MT, kv_bits):
    B, P = prompts.shape
    out = np.zeros((B, MT), np.int32)
    st = np.zeros(5, np.int64)
    assert O.lib().orc_hybrid_spec_generate(o, O.ptr(np.ascontiguousarray(prompts)), B, P, MT, kv_bits, O.ptr(out),
                                            O.ptr(st)) == 0
    return out, st
