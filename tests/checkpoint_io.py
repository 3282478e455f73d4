"""MLX-format checkpoints for the tests, in numpy: a safetensors reader and
writer (written from the format's description, independent of the library's
C++ parser), a synthetic checkpoint maker and an oracle model built from a
checkpoint -- test infrastructure.

Checkpoint layout (the reference's Qwen3 / Llama weight_map names,
src/llm/models/qwen3.cpp:100-160, :236-241): model.embed_tokens,
model.layers.{l}.self_attn.{q,k,v,o}_proj, model.layers.{l}.mlp.{gate,up,
down}_proj -- each as .weight (U32 packed), .scales, .biases -- plus
model.layers.{l}.{input,post_attention}_layernorm.weight,
model.layers.{l}.self_attn.{q,k}_norm.weight (Qwen3), model.norm.weight and
lm_head.* when the embeddings are not tied.  config.json's "quantization"
holds the default {group_size, bits} and per-layer overrides keyed by prefix.
"""
import ctypes as C
import json
import os
import struct

import numpy as np

import oracle_lib as O

PROJ = ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
        "mlp.up_proj", "mlp.down_proj"]
_NP = {"U32": np.uint32, "BF16": np.uint16, "F16": np.float16, "F32": np.float32, "I32": np.int32,
       "U8": np.uint8, "I64": np.int64}


def write_safetensors(path, tensors, metadata=None, order=None):
    """tensors: name -> (dtype string, array).  Data laid out in `order`
    (default: sorted names)."""
    names = order or sorted(tensors)
    header, off, blobs = {}, 0, []
    if metadata:
        header["__metadata__"] = metadata
    for n in names:
        dt, a = tensors[n]
        b = np.ascontiguousarray(a.astype(_NP[dt], copy=False)).tobytes()
        header[n] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_safetensors(path):
    """name -> (dtype string, array); BF16 as uint16 bit patterns."""
    with open(path, "rb") as f:
        raw = f.read()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        a, b = e["data_offsets"]
        arr = np.frombuffer(raw[8 + n + a:8 + n + b], dtype=_NP[e["dtype"]]).reshape(e["shape"])
        out[name] = (e["dtype"], arr)
    return out


def read_checkpoint(d):
    """The tensors of a model directory: shards of the index, else
    model.safetensors, else every *.safetensors (later names replace)."""
    idx = os.path.join(d, "model.safetensors.index.json")
    files = []
    if os.path.exists(idx):
        files = sorted(set(json.load(open(idx))["weight_map"].values()))
    elif os.path.exists(os.path.join(d, "model.safetensors")):
        files = ["model.safetensors"]
    else:
        files = sorted(f for f in os.listdir(d) if f.endswith(".safetensors"))
    t = {}
    for f in files:
        t.update(read_safetensors(os.path.join(d, f)))
    return t


def to_bf16(dt, a):
    if dt == "BF16":
        return a.astype(np.uint16)
    return O.f32_to_bf16(a.astype(np.float32))


def make_checkpoint(d, cfg, seed, overrides=None, norm_std=0.1, scale_dtype="BF16", shards=1,
                    model_type=None, extra=None):
    """A synthetic MLX checkpoint of `cfg` (oracle ModelCfg field names):
    linear weights N(0, 0.02) quantized at the default bits or the prefix's
    override (overrides: prefix -> bits); norms 1 + N(0, norm_std) in bf16;
    scales / biases / norms stored as scale_dtype; `shards` > 1 splits the
    tensors over files named by an index.  Returns the tensor dict."""
    overrides = overrides or {}
    H, L, I = cfg["hidden"], cfg["layers"], cfg["inter"]
    D, NQ, NK = cfg["head_dim"], cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    shapes = [(NQ, H), (NK, H), (NK, H), (H, NQ), (I, H), (I, H), (H, I)]
    t, tid = {}, 100

    def qw(prefix, N, K):
        nonlocal tid
        tid += 1
        bits = overrides.get(prefix, cfg["bits"])
        w = O.gen_normal_bf16(seed, tid, 0.02, N * K).reshape(N, K)
        wq, s, b = O.quantize(w, 64, bits)
        t[prefix + ".weight"] = ("U32", wq)
        for k, v in (("scales", s), ("biases", b)):
            t[f"{prefix}.{k}"] = (scale_dtype, O.bf16_to_f32(v) if scale_dtype != "BF16" else v)

    def nv(name, n):
        nonlocal tid
        tid += 1
        r = np.random.RandomState(seed * 1000 + tid)
        v = O.f32_to_bf16((1.0 + norm_std * r.standard_normal(n)).astype(np.float32))
        t[name] = (scale_dtype, O.bf16_to_f32(v) if scale_dtype != "BF16" else v)

    qw("model.embed_tokens", cfg["vocab"], H)
    for l in range(L):
        p = f"model.layers.{l}."
        for k in range(7):
            qw(p + PROJ[k], *shapes[k])
        nv(p + "input_layernorm.weight", H)
        nv(p + "post_attention_layernorm.weight", H)
        if cfg["qk_norm"]:
            nv(p + "self_attn.q_norm.weight", D)
            nv(p + "self_attn.k_norm.weight", D)
    nv("model.norm.weight", H)
    if not cfg["tied"]:
        qw("lm_head", cfg["vocab"], H)
    if extra:
        t.update(extra)
    os.makedirs(d, exist_ok=True)
    if shards == 1:
        write_safetensors(os.path.join(d, "model.safetensors"), t, {"format": "mlx"})
    else:
        names = sorted(t)
        wm = {}
        for i in range(shards):
            fn = f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
            part = names[i::shards]
            write_safetensors(os.path.join(d, fn), {n: t[n] for n in part})
            wm.update({n: fn for n in part})
        json.dump({"metadata": {}, "weight_map": wm}, open(os.path.join(d, "model.safetensors.index.json"), "w"))
    q = {"group_size": 64, "bits": cfg["bits"]}
    q.update({p: {"group_size": 64, "bits": b} for p, b in overrides.items()})
    conf = {"model_type": model_type or ("qwen3" if cfg["qk_norm"] else "llama"), "hidden_size": H,
            "num_hidden_layers": L, "intermediate_size": I, "num_attention_heads": cfg["heads"],
            "num_key_value_heads": cfg["kv_heads"], "head_dim": D, "vocab_size": cfg["vocab"],
            "rope_theta": cfg["rope_theta"], "rms_norm_eps": cfg["eps"],
            "tie_word_embeddings": bool(cfg["tied"]), "quantization": q, "eos_token_id": [7, 9]}
    if cfg.get("rope_factor", 0) > 1:
        conf["rope_scaling"] = {"rope_type": "llama3", "factor": cfg["rope_factor"],
                                "low_freq_factor": cfg["rope_low_freq"], "high_freq_factor": cfg["rope_high_freq"],
                                "original_max_position_embeddings": cfg["rope_orig_max_pos"]}
    json.dump(conf, open(os.path.join(d, "config.json"), "w"), indent=1)
    return t


def oracle_config(d):
    """config.json -> oracle ModelCfg kwargs (Python's json, independent of
    the library's parser)."""
    j = json.load(open(os.path.join(d, "config.json")))
    q = j.get("quantization", {})
    qwen3 = j["model_type"] == "qwen3"
    cfg = dict(hidden=j["hidden_size"], layers=j["num_hidden_layers"], inter=j["intermediate_size"],
               heads=j["num_attention_heads"], kv_heads=j.get("num_key_value_heads", j["num_attention_heads"]),
               head_dim=j.get("head_dim") or j["hidden_size"] // j["num_attention_heads"], vocab=j["vocab_size"],
               rope_theta=j.get("rope_theta", 1e6 if qwen3 else 1e4), eps=j["rms_norm_eps"], qk_norm=int(qwen3),
               tied=int(j.get("tie_word_embeddings", False)), bits=q.get("bits", 4), group=q.get("group_size", 64),
               rope_factor=0.0, rope_low_freq=0.0, rope_high_freq=0.0, rope_orig_max_pos=0.0)
    rs = j.get("rope_scaling") or {}
    if not qwen3 and rs.get("rope_type", rs.get("type")) == "llama3":
        cfg.update(rope_factor=rs.get("factor", 1.0), rope_low_freq=rs.get("low_freq_factor", 1.0),
                   rope_high_freq=rs.get("high_freq_factor", 4.0),
                   rope_orig_max_pos=rs.get("original_max_position_embeddings", 8192.0))
    return cfg, q


def oracle_from_checkpoint(d):
    """An oracle model holding the checkpoint's tensors (caller frees it)."""
    cfg, q = oracle_config(d)
    t = read_checkpoint(d)
    m = O.lib().orc_model_create(C.byref(O.ModelCfg(**cfg)), 1)
    assert m

    def put(layer, kind, prefix):
        ov = q.get(prefix)
        bits = ov.get("bits", cfg["bits"]) if isinstance(ov, dict) else cfg["bits"]
        wq = np.ascontiguousarray(t[prefix + ".weight"][1])
        s = np.ascontiguousarray(to_bf16(*t[prefix + ".scales"]))
        b = np.ascontiguousarray(to_bf16(*t[prefix + ".biases"]))
        assert O.lib().orc_model_set_weight(m, layer, kind, bits, O.ptr(wq), O.ptr(s), O.ptr(b)) == 0, prefix

    def norm(layer, which, name):
        v = np.ascontiguousarray(to_bf16(*t[name]))
        assert O.lib().orc_model_set_norm(m, layer, which, O.ptr(v)) == 0, name

    put(0, 7, "model.embed_tokens")
    for l in range(cfg["layers"]):
        p = f"model.layers.{l}."
        for k in range(7):
            put(l, k, p + PROJ[k])
        norm(l, 0, p + "input_layernorm.weight")
        norm(l, 1, p + "post_attention_layernorm.weight")
        if cfg["qk_norm"]:
            norm(l, 2, p + "self_attn.q_norm.weight")
            norm(l, 3, p + "self_attn.k_norm.weight")
    norm(0, 4, "model.norm.weight")
    if not cfg["tied"]:
        put(0, 8, "lm_head")
    return cfg, m
