"""Models loaded from MLX-format checkpoints on the B200 vs the oracle built
from the same files (by the tests' own numpy safetensors reader):
save -> load reproduces a seeded model bit for bit; synthetic checkpoints
with per-layer quantization overrides (8-bit layers in a 4-bit model, an
8-bit lm_head), non-unit norms, F16 / F32 scales and sharded files give the
oracle's logits and speculative token streams bit-exactly in exact mode and
within the tensor-core tolerance otherwise; malformed checkpoints fail with
the documented codes."""
import ctypes as C
import json
import os

import numpy as np
import pytest

import checkpoint_io as CK
import oracle_lib as O

pytestmark = pytest.mark.gpu

QWEN = dict(hidden=512, layers=3, inter=1024, heads=4, kv_heads=2, head_dim=128, vocab=1000, rope_theta=1e6,
            eps=1e-6, qk_norm=1, tied=1, bits=4, group_size=64)
LLAMA = dict(hidden=1024, layers=2, inter=2048, heads=8, kv_heads=2, head_dim=128, vocab=777, rope_theta=5e5,
             eps=1e-5, qk_norm=0, tied=0, bits=8, group_size=64, rope_factor=32.0, rope_low_freq=1.0,
             rope_high_freq=4.0, rope_orig_max_pos=8192.0)


def ocfg(cfg):
    d = dict(cfg)
    d["group"] = d.pop("group_size")
    for k in ("rope_factor", "rope_low_freq", "rope_high_freq", "rope_orig_max_pos"):
        d.setdefault(k, 0.0)
    return d


def run_blocks(lmx, g, o, cfg, kv_bits, seed, exact):
    """Prefill / verify / rollback / decode blocks on both sides; bit-exact
    logits in exact mode, else within the engine tests' tolerance."""
    L, V, B = cfg["layers"], cfg["vocab"], 2
    gc = C.c_void_p()
    lmx.call("lmx_cache_create", g.h, L, B, 160, kv_bits, 40, C.byref(gc))
    oc = O.lib().orc_cache_create(o, L, B, 160, kv_bits)
    rng = np.random.RandomState(seed)
    try:
        for i, T in enumerate([37, 5, 5, 1, 20]):
            if i == 2:
                for b, pos in enumerate([39, 38]):
                    lmx.call("lmx_cache_set_position", gc, b, pos)
                    O.lib().orc_cache_set_position(oc, b, pos)
            tok = rng.randint(0, V, (B, T)).astype(np.int32)
            gl = np.zeros((B, T, V), np.uint16)
            ol = np.zeros((B, T, V), np.uint16)
            lmx.call("lmx_forward", g.h, gc, L, tok.ctypes.data, B, T, gl.ctypes.data)
            assert O.lib().orc_forward(o, oc, L, O.ptr(tok), B, T, O.ptr(ol)) == 0
            if exact:
                bad = np.argwhere(gl != ol)
                assert bad.size == 0, f"block {i}: {len(bad)} mismatching logits, first {bad[:3].tolist()}"
            else:
                gf, of = O.bf16_to_f32(gl), O.bf16_to_f32(ol)
                diff = np.abs(gf - of)
                lim = 2e-2 + np.abs(of) * 2.0 ** -7
                assert not (diff > lim).any(), f"block {i}: max |diff| {diff.max():.4g}"
    finally:
        lmx.call("lmx_cache_free", gc)
        O.lib().orc_cache_free(oc)


@pytest.mark.parametrize("cfg", [QWEN, LLAMA], ids=["qwen3-4bit-tied", "llama-8bit-rope-scaled"])
def test_save_load_reproduces_seeded_model(lmx, cuda, mma_threshold, tmp_path, cfg):
    mma_threshold(0)
    g = lmx.Model(cfg, 4242)
    d = str(tmp_path / "ck")
    g.save(d)
    got_cfg, eos = lmx.config_load(d)
    for k, v in cfg.items():
        assert got_cfg[k] == pytest.approx(v), k
    # the file holds exactly the device tensors (numpy reader)
    t = CK.read_checkpoint(d)
    H, D, bits = cfg["hidden"], cfg["head_dim"], cfg["bits"]
    w = np.zeros((H, cfg["inter"] * bits // 32), np.uint32)
    s = np.zeros((H, cfg["inter"] // 64), np.uint16)
    b = np.zeros_like(s)
    lmx.call("lmx_model_weight", g.h, 1, 6, w.ctypes.data, s.ctypes.data, b.ctypes.data)
    np.testing.assert_array_equal(t["model.layers.1.mlp.down_proj.weight"][1], w)
    np.testing.assert_array_equal(t["model.layers.1.mlp.down_proj.scales"][1], s)
    np.testing.assert_array_equal(t["model.layers.1.mlp.down_proj.biases"][1], b)
    assert ("lm_head.weight" in t) == (not cfg["tied"])
    assert ("model.layers.0.self_attn.q_norm.weight" in t) == bool(cfg["qk_norm"])
    g2 = lmx.Model.load(d)
    L, V, B, T = cfg["layers"], cfg["vocab"], 2, 12
    tok = np.random.RandomState(2).randint(0, V, (B, T)).astype(np.int32)
    outs = []
    for m in (g, g2):
        gc = C.c_void_p()
        lmx.call("lmx_cache_create", m.h, L, B, 64, 16, T, C.byref(gc))
        lg = np.zeros((B, T, V), np.uint16)
        lmx.call("lmx_forward", m.h, gc, L, tok.ctypes.data, B, T, lg.ctypes.data)
        lmx.call("lmx_cache_free", gc)
        outs.append(lg)
    np.testing.assert_array_equal(outs[0], outs[1])
    g2.close()
    g.close()


CASES = {
    # 8-bit o_proj / down_proj in one layer and an 8-bit lm_head in a 4-bit
    # model; non-unit norms; BF16 scales
    "qwen3-mixed": (dict(QWEN, tied=0), {"model.layers.1.self_attn.o_proj": 8, "model.layers.1.mlp.down_proj": 8,
                                        "model.layers.2.mlp.gate_proj": 8, "model.layers.2.mlp.up_proj": 8,
                                        "lm_head": 8}, "BF16", 1),
    # 8-bit tied embedding (lookup and lm_head) and q/k/v of layer 0;
    # F16 scales and norms rounded to bf16 on load; three shards
    "qwen3-tied8-f16-shards": (QWEN, {"model.embed_tokens": 8, "model.layers.0.self_attn.q_proj": 8,
                                      "model.layers.0.self_attn.k_proj": 8, "model.layers.0.self_attn.v_proj": 8},
                               "F16", 3),
    # Llama, 8-bit default with a 4-bit layer, F32 scales
    "llama-8bit-f32": (LLAMA, {"model.layers.0.mlp.down_proj": 4}, "F32", 1),
}


@pytest.fixture(scope="module")
def loaded(lmx, cuda, tmp_path_factory):
    out = {}
    for name, (cfg, over, sdt, shards) in CASES.items():
        d = str(tmp_path_factory.mktemp(name))
        CK.make_checkpoint(d, ocfg(cfg), 31, overrides=over, scale_dtype=sdt, shards=shards)
        g = lmx.Model.load(d)
        _, o = CK.oracle_from_checkpoint(d)
        out[name] = (cfg, g, o, d)
    yield out
    for cfg, g, o, d in out.values():
        g.close()
        O.lib().orc_model_free(o)


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("kv_bits", [16, 8])
def test_checkpoint_forward_bit_exact(lmx, loaded, mma_threshold, name, kv_bits):
    mma_threshold(0)
    cfg, g, o, _ = loaded[name]
    run_blocks(lmx, g, o, cfg, kv_bits, 11, exact=True)


@pytest.mark.parametrize("name", list(CASES))
def test_checkpoint_forward_tensor_core(lmx, loaded, mma_threshold, name):
    # blocks of >= 16 rows on tcgen05 (the oracle emulates the same form)
    mma_threshold(16)
    cfg, g, o, _ = loaded[name]
    run_blocks(lmx, g, o, cfg, 16, 12, exact=False)


@pytest.mark.parametrize("name", ["qwen3-mixed", "qwen3-tied8-f16-shards"])
def test_checkpoint_spec_stream_bit_exact(lmx, loaded, mma_threshold, name):
    # self-draft (first layer) speculative decoding of the loaded model
    mma_threshold(0)
    cfg, g, o, _ = loaded[name]
    B, P, K, MT = 2, 16, 3, 40
    prompts = np.random.RandomState(5).randint(0, cfg["vocab"], (B, P)).astype(np.int32)
    sd = lmx.SpecDecoder(g, None, 1, B, K, MT, P, kv_bits=16)
    sd.prefill(prompts)
    sd.decode(use_graph=True)
    got, _ = sd.result()
    sd.close()
    ref = np.zeros((B, MT), np.int32)
    st = np.zeros(5, np.int64)
    prm = O.SpecParams(K=K, max_tokens=MT, temperature=0.0, top_p=1.0, seed=0, draft_layers=1)
    assert O.lib().orc_spec_generate(o, None, O.ptr(prompts), B, P, prm, 16, O.ptr(ref), O.ptr(st)) == 0
    np.testing.assert_array_equal(got, ref)


def test_fused_decode_skips_mixed_precision(lmx, loaded, mma_threshold):
    # the fused decode kernel takes one bits value for every weight: a mixed
    # checkpoint runs the per-op path even with the switch on (same logits)
    mma_threshold(16)
    cfg, g, o, _ = loaded["qwen3-mixed"]
    lmx.call("lmx_set_fused_decode", 1)
    try:
        run_blocks(lmx, g, o, cfg, 16, 13, exact=False)
    finally:
        lmx.call("lmx_set_fused_decode", 0)


def load_rc(lmx, d):
    h = C.c_void_p()
    rc = lmx.lib().lmx_model_load(os.fsencode(d), C.byref(h))
    if rc == 0:
        lmx.lib().lmx_model_free(h)
    return rc, lmx.lib().lmx_last_error()


def test_checkpoint_errors(lmx, cuda, tmp_path):
    cfg = ocfg(QWEN)
    base = str(tmp_path / "base")
    t = CK.make_checkpoint(base, cfg, 3)
    conf = json.load(open(os.path.join(base, "config.json")))

    def variant(name, tensors, conf_=None):
        d = tmp_path / name
        d.mkdir()
        CK.write_safetensors(str(d / "model.safetensors"), tensors)
        (d / "config.json").write_text(json.dumps(conf_ or conf))
        return str(d)

    missing = {k: v for k, v in t.items() if k != "model.layers.2.mlp.up_proj.biases"}
    rc, msg = load_rc(lmx, variant("missing", missing))
    assert rc == 2 and b"model.layers.2.mlp.up_proj" in msg, msg
    missing = {k: v for k, v in t.items() if k != "model.layers.1.post_attention_layernorm.weight"}
    rc, msg = load_rc(lmx, variant("missing_norm", missing))
    assert rc == 6 and b"post_attention_layernorm" in msg, msg
    unq = {k: v for k, v in t.items() if not k.startswith("model.layers.0.self_attn.o_proj.")}
    unq["model.layers.0.self_attn.o_proj.weight"] = ("BF16", np.zeros((512, 512), np.uint16))
    rc, msg = load_rc(lmx, variant("unquantized", unq))
    assert rc == 2 and b"not quantized" in msg, msg
    rc, msg = load_rc(lmx, variant("shape", t, dict(conf, intermediate_size=2048)))
    assert rc == 6 and b"expected U32" in msg, msg
    q = dict(conf["quantization"], **{"model.layers.0.self_attn.k_proj": {"bits": 8, "group_size": 64}})
    rc, msg = load_rc(lmx, variant("qkv_bits", t, dict(conf, quantization=q)))
    assert rc == 6 and b"expected U32" in msg, msg  # the file's k_proj is 4-bit: width disagrees
    rc, msg = load_rc(lmx, variant("noquant", t, {k: v for k, v in conf.items() if k != "quantization"}))
    assert rc == 2 and b"quantization" in msg, msg
    rc, msg = load_rc(lmx, str(tmp_path / "none"))
    assert rc == 6, msg


def test_mixed_qkv_bits_rejected(lmx, cuda, tmp_path):
    # q/k/v run as one fused GEMM: a checkpoint that quantizes them
    # differently is refused with a clear message
    d = str(tmp_path / "ck")
    CK.make_checkpoint(d, ocfg(QWEN), 9, overrides={"model.layers.1.self_attn.v_proj": 8})
    rc, msg = load_rc(lmx, d)
    assert rc == 2 and b"share their bits" in msg, msg
