"""Checkpoint handling on the host (no GPU): config.json parsing with the
reference's defaults and per-layer quantization lookup
(parse_base_configuration, src/common/base_config.cpp:9-73;
quantization_for, include/mlx-lm/common/base_config.h:47-54; Qwen3 / Llama
from_json, src/llm/models/qwen3.cpp:13-35, llama.cpp:22-55), the safetensors
header parser against files written by an independent numpy writer, its
rejection of malformed files, and the oracle built from a checkpoint."""
import ctypes as C
import json
import os
import struct

import numpy as np
import pytest

import checkpoint_io as CK
import oracle_lib as O

QWEN = {"model_type": "qwen3", "hidden_size": 1024, "num_hidden_layers": 28, "intermediate_size": 3072,
        "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 151936,
        "rms_norm_eps": 1e-06, "rope_theta": 1000000, "tie_word_embeddings": True, "eos_token_id": 151645,
        "quantization": {"group_size": 64, "bits": 4, "mode": "affine",
                         "model.layers.3.mlp.down_proj": {"group_size": 64, "bits": 8},
                         "language_model.model.layers.5.self_attn.v_proj": {"bits": 8, "group_size": 64},
                         "model.layers.7.mlp.gate_proj": False}}
LLAMA = {"model_type": "llama", "hidden_size": 2048, "num_hidden_layers": 16, "intermediate_size": 8192,
         "num_attention_heads": 32, "num_key_value_heads": 8, "vocab_size": 128256, "rms_norm_eps": 1e-05,
         "rope_theta": 500000.0, "tie_word_embeddings": True, "eos_token_id": [128001, 128008, 128009],
         "rope_scaling": {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0,
                          "original_max_position_embeddings": 8192, "rope_type": "llama3"},
         "quantization": {"group_size": 64, "bits": 8}}


def write_cfg(tmp_path, j, name="config.json"):
    p = tmp_path / name
    p.write_text(json.dumps(j) if not isinstance(j, str) else j)
    return str(tmp_path)


def load(lmx, path):
    c = lmx.ModelConfig()
    eos = (C.c_int32 * 8)()
    n = C.c_int()
    rc = lmx.lib().lmx_model_config_load(os.fsencode(path), C.byref(c), eos, 8, C.byref(n))
    return rc, c, list(eos[:min(n.value, 8)])


def test_qwen3_config_and_quant_overrides(lmx, tmp_path):
    d = write_cfg(tmp_path, QWEN)
    rc, c, eos = load(lmx, d)
    assert rc == 0, lmx.lib().lmx_last_error()
    assert (c.hidden, c.layers, c.inter, c.heads, c.kv_heads, c.head_dim, c.vocab) == \
        (1024, 28, 3072, 16, 8, 128, 151936)
    assert c.qk_norm == 1 and c.tied == 1 and c.bits == 4 and c.group_size == 64 and c.rope_factor == 0
    assert c.rope_theta == 1e6 and c.eps == np.float32(1e-6)
    assert eos == [151645]

    def qf(prefix):
        b, g = C.c_int(), C.c_int()
        assert lmx.lib().lmx_model_quant_for(os.fsencode(d), prefix.encode(), C.byref(b), C.byref(g)) == 0
        return b.value, g.value

    assert qf("model.layers.3.mlp.down_proj") == (8, 64)
    assert qf("model.layers.5.self_attn.v_proj") == (8, 64)  # "language_model." stripped
    assert qf("model.layers.7.mlp.gate_proj") == (4, 64)     # `false`: the default (quantization_for)
    assert qf("model.layers.3.mlp.up_proj") == (4, 64)
    assert qf("model.layers.3") == (4, 64)                   # exact prefixes only


def test_llama_config_defaults_and_rope_scaling(lmx, tmp_path):
    d = write_cfg(tmp_path, LLAMA)
    rc, c, eos = load(lmx, d)
    assert rc == 0, lmx.lib().lmx_last_error()
    # head_dim absent: hidden / heads; no q/k norm; llama3 frequency scaling
    assert c.head_dim == 64 and c.qk_norm == 0 and c.bits == 8 and c.tied == 1
    assert (c.rope_factor, c.rope_low_freq, c.rope_high_freq, c.rope_orig_max_pos) == (32.0, 1.0, 4.0, 8192.0)
    assert eos == [128001, 128008, 128009]
    j = dict(LLAMA)
    del j["num_key_value_heads"], j["rope_theta"]
    j["rope_scaling"] = {"rope_type": "llama3"}  # every field defaulted (compute_freqs)
    j["text_config"] = {"eos_token_id": 5}
    del j["eos_token_id"]
    rc, c, eos = load(lmx, write_cfg(tmp_path, j))
    assert rc == 0 and c.kv_heads == 32 and c.rope_theta == 10000.0 and eos == [5]
    assert (c.rope_factor, c.rope_low_freq, c.rope_high_freq, c.rope_orig_max_pos) == (1.0, 1.0, 4.0, 8192.0)


@pytest.mark.parametrize("bad,code,msg", [
    ('{"model_type": "qwen3", "hidden_size": 10', 6, b"malformed"),
    ('{"model_type": "qwen3"} x', 6, b"trailing"),
    ('{"model_type": "gpt2", "hidden_size": 1}', 2, b"gpt2"),
    ('{"model_type": "qwen3", "hidden_size": 1024}', 6, b"num_hidden_layers"),
    ('{"a": "\\ud800"}', 6, b"surrogate"),
    ('[' * 100 + ']' * 100, 6, b"deep"),
])
def test_config_errors(lmx, tmp_path, bad, code, msg):
    rc, _, _ = load(lmx, write_cfg(tmp_path, bad))
    assert rc == code and msg in lmx.lib().lmx_last_error(), lmx.lib().lmx_last_error()


def test_config_rejects_unsupported_features(lmx, tmp_path):
    for extra in ({"attention_bias": True}, {"rope_traditional": True},
                  {"quantization": {"group_size": 32, "bits": 4, "mode": "mxfp4"}}):
        rc, _, _ = load(lmx, write_cfg(tmp_path, dict(LLAMA, **extra)))
        assert rc == 2, lmx.lib().lmx_last_error()
    rc, _, _ = load(lmx, str(tmp_path / "nowhere"))
    assert rc == 6 and b"config.json not found" in lmx.lib().lmx_last_error()


def test_json_escapes_and_numbers(lmx, tmp_path):
    # keys with escapes / unicode, exponents, whitespace everywhere
    j = ' { "model_type" : "qw\\u0065n3" , "hidden_size":1.024e3,"num_hidden_layers":2,"intermediate_size":512,' \
        '"num_attention_heads":4,"num_key_value_heads":2,"head_dim":128,"vocab_size":1000,' \
        '"rms_norm_eps":1E-6,"x\\"\\\\\\/\\b\\f\\n\\r\\t\\u00e9\\ud83d\\ude00":[true,false,null,-0.5e-3,{}],' \
        '"quantization":{"bits":8}}\n'
    rc, c, _ = load(lmx, write_cfg(tmp_path, j))
    assert rc == 0, lmx.lib().lmx_last_error()
    assert c.hidden == 1024 and c.bits == 8 and c.group_size == 64 and c.eps == np.float32(1e-6)


def st_info(lmx, path, name):
    dt = C.create_string_buffer(16)
    shape = (C.c_int64 * 8)()
    nd = C.c_int()
    off = C.c_uint64()
    rc = lmx.lib().lmx_safetensors_tensor(os.fsencode(path), name.encode(), dt, shape, 8, C.byref(nd), C.byref(off))
    return rc, dt.value.decode(), list(shape[:nd.value]), off.value


def test_safetensors_header_parse(lmx, tmp_path):
    rng = np.random.RandomState(3)
    t = {"a.weight": ("U32", rng.randint(0, 2**32, (5, 8), dtype=np.uint64).astype(np.uint32)),
         "a.scales": ("BF16", rng.randint(0, 2**16, (5, 2)).astype(np.uint16)),
         "né": ("F32", rng.standard_normal(7).astype(np.float32)),
         "empty": ("F16", np.zeros((0, 3), np.float16)),
         "scalar": ("I32", np.array(42, np.int32))}
    p = str(tmp_path / "x.safetensors")
    CK.write_safetensors(p, t, {"format": "mlx"}, order=["né", "a.weight", "empty", "scalar", "a.scales"])
    raw = open(p, "rb").read()
    for name, (dt, a) in t.items():
        rc, gdt, shape, off = st_info(lmx, p, name)
        assert rc == 0, lmx.lib().lmx_last_error()
        assert gdt == dt and shape == list(a.shape)
        nb = a.nbytes
        assert raw[off:off + nb] == np.ascontiguousarray(a).tobytes()
    rc, *_ = st_info(lmx, p, "missing")
    assert rc == 1 and b"no tensor" in lmx.lib().lmx_last_error()


def test_safetensors_rejects_malformed(lmx, tmp_path):
    good = str(tmp_path / "g.safetensors")
    CK.write_safetensors(good, {"w": ("F32", np.ones((4, 4), np.float32))})
    raw = open(good, "rb").read()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])

    def variant(name, hdr=None, body=None, hlen=None):
        h = json.dumps(hdr if hdr is not None else header).encode()
        p = str(tmp_path / name)
        with open(p, "wb") as f:
            f.write(struct.pack("<Q", hlen if hlen is not None else len(h)))
            f.write(h)
            f.write(raw[8 + n:] if body is None else body)
        return p

    cases = [
        variant("trunc.st", body=raw[8 + n:-4]),                                   # data cut short
        variant("shape.st", hdr={"w": dict(header["w"], shape=[4, 5])}),           # shape vs offsets
        variant("dtype.st", hdr={"w": dict(header["w"], dtype="Q7")}),             # unknown dtype
        variant("order.st", hdr={"w": dict(header["w"], data_offsets=[64, 0])}),  # end < begin
        variant("hlen.st", hlen=1 << 40),                                          # header past the file
        variant("neg.st", hdr={"w": dict(header["w"], shape=[-4, -4])}),
    ]
    for p in cases:
        rc, *_ = st_info(lmx, p, "w")
        assert rc == 6, (p, lmx.lib().lmx_last_error())
    tiny = str(tmp_path / "tiny.st")
    open(tiny, "wb").write(b"\x01\x00")
    assert st_info(lmx, tiny, "w")[0] == 6


TINY = dict(hidden=512, layers=2, inter=1024, heads=4, kv_heads=2, head_dim=128, vocab=500, rope_theta=1e6,
            eps=1e-6, qk_norm=1, tied=0, bits=4, group=64, rope_factor=0.0, rope_low_freq=0.0, rope_high_freq=0.0,
            rope_orig_max_pos=0.0)


def oracle_logits(o, cfg, tok):
    B, T = tok.shape
    oc = O.lib().orc_cache_create(o, cfg["layers"], B, 64, 16)
    out = np.zeros((B, T, cfg["vocab"]), np.uint16)
    assert O.lib().orc_forward(o, oc, cfg["layers"], O.ptr(tok), B, T, O.ptr(out)) == 0
    O.lib().orc_cache_free(oc)
    return out


def test_oracle_from_checkpoint_reproduces_seeded_model(tmp_path):
    # export a seeded oracle model's tensors as a checkpoint, rebuild an
    # oracle model from the file: identical logits
    o = O.lib().orc_model_create(C.byref(O.ModelCfg(**TINY)), 77)
    H, D, I, V = TINY["hidden"], TINY["head_dim"], TINY["inter"], TINY["vocab"]
    shapes = [(4 * D, H), (2 * D, H), (2 * D, H), (H, 4 * D), (I, H), (I, H), (H, I)]
    t = {}

    def grab(layer, kind, prefix, N, K):
        w = np.zeros((N, K // 8), np.uint32)
        s = np.zeros((N, K // 64), np.uint16)
        b = np.zeros_like(s)
        assert O.lib().orc_model_weight(o, layer, kind, O.ptr(w), O.ptr(s), O.ptr(b)) == 0
        t.update({prefix + ".weight": ("U32", w), prefix + ".scales": ("BF16", s), prefix + ".biases": ("BF16", b)})

    ones = lambda n: ("BF16", np.full(n, 0x3F80, np.uint16))
    grab(0, 7, "model.embed_tokens", V, H)
    grab(0, 8, "lm_head", V, H)
    for l in range(2):
        for k in range(7):
            grab(l, k, f"model.layers.{l}.{CK.PROJ[k]}", *shapes[k])
        for n, sz in (("input_layernorm", H), ("post_attention_layernorm", H), ("self_attn.q_norm", D),
                      ("self_attn.k_norm", D)):
            t[f"model.layers.{l}.{n}.weight"] = ones(sz)
    t["model.norm.weight"] = ones(H)
    d = tmp_path / "ck"
    d.mkdir()
    CK.write_safetensors(str(d / "model.safetensors"), t)
    conf = {"model_type": "qwen3", "hidden_size": H, "num_hidden_layers": 2, "intermediate_size": I,
            "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": D, "vocab_size": V,
            "rms_norm_eps": 1e-6, "rope_theta": 1e6, "tie_word_embeddings": False,
            "quantization": {"group_size": 64, "bits": 4}}
    (d / "config.json").write_text(json.dumps(conf))
    cfg, o2 = CK.oracle_from_checkpoint(str(d))
    tok = np.random.RandomState(1).randint(0, V, (2, 9)).astype(np.int32)
    np.testing.assert_array_equal(oracle_logits(o, TINY, tok), oracle_logits(o2, TINY, tok))
    O.lib().orc_model_free(o)
    O.lib().orc_model_free(o2)


def test_checkpoint_maker_roundtrip(tmp_path):
    # the numpy writer / reader agree, shards and F16 scales included, and the
    # override reaches the weight's packed width
    cfg = dict(TINY, tied=1)
    d = str(tmp_path / "ck")
    t = CK.make_checkpoint(d, cfg, 5, overrides={"model.layers.1.mlp.down_proj": 8}, scale_dtype="F16", shards=3)
    back = CK.read_checkpoint(d)
    assert set(back) == set(t)
    for n, (dt, a) in t.items():
        assert back[n][0] == dt
        np.testing.assert_array_equal(back[n][1], a.astype(back[n][1].dtype))
    assert back["model.layers.1.mlp.down_proj.weight"][1].shape == (512, 1024 * 8 // 32)
    assert back["model.layers.0.mlp.down_proj.weight"][1].shape == (512, 1024 * 4 // 32)
    assert "lm_head.weight" not in back
    cfg2, o = CK.oracle_from_checkpoint(d)
    assert cfg2["tied"] == 1 and cfg2["bits"] == 4
    O.lib().orc_model_free(o)
