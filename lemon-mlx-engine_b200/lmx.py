"""ctypes binding of liblmx.so, the B200 speculative-decode library.

This is a thin host-side mirror of the C ABI in include/lmx.h.  It never
falls back to another implementation: if the CUDA library is missing or a call
fails, it raises.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblmx.so")

P = C.c_void_p
I = C.c_int
I64 = C.c_int64
U64 = C.c_uint64
F = C.c_float

_lib = None


class LmxError(RuntimeError):
    pass


# Every exported symbol of include/lmx.h with (restype, argtypes).
SIGNATURES = {
    "lmx_last_error": (C.c_char_p, []),
    "lmx_version": (C.c_char_p, []),
    "lmx_set_device": (I, [I]),
    "lmx_device_error": (I, [C.POINTER(C.c_uint), I]),
    "lmx_quantized_matmul": (I, [P, P, P, P, P, I, I, I, I, I, P]),
    "lmx_set_mma_min_m": (I, [I]),
    "lmx_launch_count": (C.c_longlong, []),
    "lmx_mma_min_m": (I, []),
    "lmx_set_gemv_tc_min_m": (I, [I]),
    "lmx_gemv_tc_min_m": (I, []),
    "lmx_set_gemm_tcs_max_m": (I, [I]),
    "lmx_gemm_tcs_max_m": (I, []),
    "lmx_set_gemv_tc_rows_min_tiles": (I, [I]),
    "lmx_gemv_tc_rows_min_tiles": (I, []),
    "lmx_set_fused_decode": (I, [I]),
    "lmx_fused_decode": (I, []),
    "lmx_set_sdpa_tc_min_cache": (I, [I]),
    "lmx_sdpa_tc_min_cache": (I, []),
    "lmx_rms_norm": (I, [P, P, P, I, I, F, P]),
    "lmx_argmax": (I, [P, I, I, P, P]),
    "lmx_sample": (I, [P, I, I, F, F, P, P, P]),
    "lmx_spec_accept": (I, [P, P, P, I, I, I, F, F, P, P, P, P, P]),
    "lmx_sdpa_scratch_bytes": (C.c_size_t, [I, I, I, I, I]),
    "lmx_sdpa_decode": (I, [P, P, I, I, F, P, C.c_size_t, P, P]),
    "lmx_sdpa_decode_noalloc": (I, [P, P, I, I, F, P, P]),
    "lmx_kv_append": (I, [P, P, P, I, P]),
    "lmx_kv_set_position": (I, [P, I, I, P]),
    "lmx_cache_kv": (I, [P, I, P]),
    "lmx_model_create": (I, [P, U64, P]),
    "lmx_model_create_tp": (I, [P, U64, P, P]),
    "lmx_model_config_load": (I, [C.c_char_p, P, P, I, P]),
    "lmx_model_quant_for": (I, [C.c_char_p, C.c_char_p, P, P]),
    "lmx_safetensors_tensor": (I, [C.c_char_p, C.c_char_p, C.c_char_p, P, I, P, P]),
    "lmx_model_load": (I, [C.c_char_p, P]),
    "lmx_model_load_tp": (I, [C.c_char_p, P, P]),
    "lmx_model_save": (I, [P, C.c_char_p]),
    "lmx_tp_comm_create": (I, [I, I, I, I, P]),
    "lmx_tp_comm_handle": (I, [P, P]),
    "lmx_tp_comm_open": (I, [P, P]),
    "lmx_tp_comm_free": (I, [P]),
    "lmx_tp_comm_block_bytes": (C.c_size_t, [P]),
    "lmx_tp_comm_attach": (I, [P, I, P]),
    "lmx_tp_comm_partial": (I, [P, P]),
    "lmx_tp_allreduce_rmsnorm": (I, [P, P, I, I, P, P, F, P, P]),
    "lmx_cache_fill_synthetic": (I, [P, I, U64, C.c_uint32]),
    "lmx_gdn_scratch_bytes": (C.c_size_t, [I, I, I, I]),
    "lmx_set_gdn_state_bf16": (I, [I]),
    "lmx_gdn_state_bf16": (I, []),
    "lmx_gdn_verify": (I, [P, P]),
    "lmx_gdn_commit": (I, [P, P, P]),
    "lmx_moe_route": (I, [P, I, I, I, P, P, P]),
    "lmx_moe_experts": (I, [P, I, I, I, I, I, P, P, P, P, P, I, P, P, P]),
    "lmx_hybrid_create": (I, [P, U64, P]),
    "lmx_hybrid_create_ep": (I, [P, U64, P, P]),
    "lmx_hybrid_free": (I, [P]),
    "lmx_hybrid_state_create": (I, [P, I, I, I, I, P]),
    "lmx_hybrid_state_free": (I, [P]),
    "lmx_hybrid_forward": (I, [P, P, P, I, I, P]),
    "lmx_hybrid_spec_create": (I, [P, I, I, I, I, P]),
    "lmx_hybrid_spec_prefill": (I, [P, P]),
    "lmx_hybrid_spec_decode": (I, [P, I, P]),
    "lmx_hybrid_spec_result": (I, [P, P, P]),
    "lmx_hybrid_spec_free": (I, [P]),
    "lmx_hybrid_spec_profile": (I, [P, I, P, P]),
    "lmx_hybrid_spec_step_launches": (I, [P, P]),
    "lmx_model_view": (I, [P, I, P]),
    "lmx_model_free": (I, [P]),
    "lmx_model_weight": (I, [P, I, I, P, P, P]),
    "lmx_cache_create": (I, [P, I, I, I, I, I, P]),
    "lmx_cache_free": (I, [P]),
    "lmx_cache_set_position": (I, [P, I, I]),
    "lmx_cache_len": (I, [P, I, P]),
    "lmx_forward": (I, [P, P, I, P, I, I, P]),
    "lmx_spec_create": (I, [P, P, I, P, P]),
    "lmx_spec_prefill": (I, [P, P]),
    "lmx_spec_decode": (I, [P, I, P]),
    "lmx_spec_result": (I, [P, P, P]),
    "lmx_spec_free": (I, [P]),
    "lmx_spec_next": (I, [P, P, P]),
    "lmx_spec_generate": (I, [P, P, P, I, P, P, P, P, P]),
    "lmx_spec_profile": (I, [P, I, I, P, P]),
    "lmx_spec_step_launches": (I, [P, P]),
}


class KvDesc(C.Structure):
    """lmx_kv"""
    _fields_ = [("batch", I), ("kv_heads", I), ("head_dim", I), ("capacity", I), ("bits", I),
                ("k", P), ("v", P), ("k_packed", P), ("v_packed", P), ("k_scales", P),
                ("k_biases", P), ("v_scales", P), ("v_biases", P), ("lengths", P)]


class GdnDesc(C.Structure):
    """lmx_gdn"""
    _fields_ = [("batch", I), ("T", I), ("k_heads", I), ("v_heads", I), ("qkv", P), ("z", P), ("b", P),
                ("a", P), ("conv_w", P), ("a_log", P), ("dt_bias", P), ("norm_w", P), ("eps", F),
                ("conv_state", P), ("state", P), ("state_snap", P), ("out", P), ("scratch", P)]


class QWeights(C.Structure):
    """lmx_qweights"""
    _fields_ = [("w", P), ("scales", P), ("biases", P)]


class HybridConfig(C.Structure):
    """lmx_hybrid_config"""
    _fields_ = [("hidden", I), ("layers", I), ("attn_every", I), ("heads", I), ("kv_heads", I),
                ("lin_k_heads", I), ("lin_v_heads", I), ("experts", I), ("top_k", I), ("expert_inter", I),
                ("shared_inter", I), ("vocab", I), ("rope_theta", F), ("eps", F), ("bits", I)]


class ModelConfig(C.Structure):
    """lmx_model_config"""
    _fields_ = [("hidden", I), ("layers", I), ("inter", I), ("heads", I), ("kv_heads", I),
                ("head_dim", I), ("vocab", I), ("rope_theta", F), ("eps", F), ("qk_norm", I),
                ("tied", I), ("bits", I), ("group_size", I), ("rope_factor", F), ("rope_low_freq", F),
                ("rope_high_freq", F), ("rope_orig_max_pos", F)]


class SpecConfig(C.Structure):
    """lmx_spec_config"""
    _fields_ = [("batch", I), ("K", I), ("max_tokens", I), ("prompt_len", I), ("kv_bits", I),
                ("temperature", F), ("top_p", F), ("seed", U64), ("context_len", I),
                ("context_seed", U64), ("seq_base", I), ("kv_quirk", I)]


# Qwen3-Next-style hybrid (the unspecified head counts / dims
# chosen: 16 q / 2 kv attention heads and 16 key / 32 value Gated DeltaNet
# heads, all of dim 128; RoPE theta 1e7 over the full head).
QWEN3_NEXT_HYBRID = dict(hidden=2048, layers=48, attn_every=4, heads=16, kv_heads=2, lin_k_heads=16,
                         lin_v_heads=32, experts=512, top_k=10, expert_inter=512, shared_inter=512,
                         vocab=151936, rope_theta=1e7, eps=1e-6, bits=4)

# The benchmark configurations' architectures (random-initialised weights).
QWEN3_0_6B = dict(hidden=1024, layers=28, inter=3072, heads=16, kv_heads=8, head_dim=128,
                  vocab=151936, rope_theta=1e6, eps=1e-6, qk_norm=1, tied=1, bits=4, group_size=64)
QWEN3_8B = dict(hidden=4096, layers=36, inter=12288, heads=32, kv_heads=8, head_dim=128,
                vocab=151936, rope_theta=1e6, eps=1e-6, qk_norm=1, tied=0, bits=4, group_size=64)
LLAMA3_70B = dict(hidden=8192, layers=80, inter=28672, heads=64, kv_heads=8, head_dim=128,
                  vocab=128256, rope_theta=5e5, eps=1e-5, qk_norm=0, tied=0, bits=4, group_size=64)
LLAMA32_1B = dict(hidden=2048, layers=16, inter=8192, heads=32, kv_heads=8, head_dim=128,
                  vocab=128256, rope_theta=5e5, eps=1e-5, qk_norm=0, tied=1, bits=4, group_size=64,
                  rope_factor=32.0, rope_low_freq=1.0, rope_high_freq=4.0, rope_orig_max_pos=8192.0)


TP_HANDLE_BYTES = 64


def exchange_handles(handle: bytes, group=None):
    """All ranks' communicator handles in rank order, gathered over an
    initialised torch.distributed process group (any backend)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    for i, h in enumerate(out):
        if not isinstance(h, bytes) or len(h) != TP_HANDLE_BYTES:
            raise LmxError(f"tp handle of rank {i} is malformed")
    return out


class TpComm:
    """Tensor-parallel communicator of this rank (include/lmx.h, 'Tensor
    parallelism'): an IPC-exported device block, opened by every peer."""

    def __init__(self, rank: int, size: int, max_rows: int, max_hidden: int):
        h = C.c_void_p()
        call("lmx_tp_comm_create", rank, size, max_rows, max_hidden, C.byref(h))
        self.h, self.rank, self.size = h, rank, size
        self._models = []

    def handle(self) -> bytes:
        buf = C.create_string_buffer(TP_HANDLE_BYTES)
        call("lmx_tp_comm_handle", self.h, buf)
        return buf.raw

    def open(self, handles):
        if len(handles) != self.size:
            raise LmxError(f"tp_comm_open: {len(handles)} handles for size {self.size}")
        blob = b"".join(handles)
        call("lmx_tp_comm_open", self.h, C.c_char_p(blob))

    @classmethod
    def from_process_group(cls, max_rows: int, max_hidden: int, group=None):
        """Create, exchange handles over torch.distributed, open, barrier."""
        import torch.distributed as dist
        rank, size = dist.get_rank(group), dist.get_world_size(group)
        comm = cls(rank, size, max_rows, max_hidden)
        if size > 1:
            comm.open(exchange_handles(comm.handle(), group))
        dist.barrier(group)
        return comm

    def close(self):
        if self.h:
            lib().lmx_tp_comm_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """Owns an lmx model handle (synthetic seeded weights on the device);
    with a TpComm of size > 1, this rank's tensor-parallel shard."""

    def __init__(self, cfg: dict, seed: int, _handle=None, _parent=None, comm=None):
        self.cfg = dict(cfg)
        self._parent = _parent
        self._comm = comm
        if _handle is not None:
            self.h = _handle
            return
        h = C.c_void_p()
        if comm is not None:
            call("lmx_model_create_tp", C.byref(ModelConfig(**cfg)), seed, comm.h, C.byref(h))
        else:
            call("lmx_model_create", C.byref(ModelConfig(**cfg)), seed, C.byref(h))
        self.h = h

    @classmethod
    def load(cls, path: str, comm=None):
        """An MLX-format checkpoint directory (config.json + safetensors);
        with a TpComm of size > 1, this rank's shard."""
        cfg = config_load(path)[0]
        h = C.c_void_p()
        if comm is not None:
            call("lmx_model_load_tp", os.fsencode(path), comm.h, C.byref(h))
        else:
            call("lmx_model_load", os.fsencode(path), C.byref(h))
        m = cls(cfg, 0, _handle=h)
        m._comm = comm
        return m

    def save(self, path: str):
        call("lmx_model_save", self.h, os.fsencode(path))

    def view(self, n_layers):
        h = C.c_void_p()
        call("lmx_model_view", self.h, n_layers, C.byref(h))
        cfg = dict(self.cfg, layers=n_layers)
        return Model(cfg, 0, _handle=h, _parent=self)

    def close(self):
        if self.h:
            lib().lmx_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def config_load(path: str):
    """config.json (file or directory) -> (lmx_model_config as a dict, EOS ids)."""
    c = ModelConfig()
    eos = (C.c_int32 * 16)()
    n = C.c_int()
    call("lmx_model_config_load", os.fsencode(path), C.byref(c), eos, 16, C.byref(n))
    return {f: getattr(c, f) for f, _ in ModelConfig._fields_}, list(eos[:min(n.value, 16)])


class CompletionInfo(C.Structure):
    """lmx_completion_info (GenerateCompletionInfo)"""
    _fields_ = [("prompt_token_count", I), ("generation_token_count", I), ("prompt_time", C.c_double),
                ("generation_time", C.c_double), ("mtp_draft_tokens_proposed", I),
                ("mtp_draft_tokens_accepted", I), ("mtp_speculative_steps", I)]


CANCEL_FN = C.CFUNCTYPE(C.c_int, C.c_void_p)
TOKEN_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.c_int32)


class SpecDecoder:
    """Speculative decoder over a target and a draft (or self-draft) model:
    the reference's generate()/TokenIterator emission contract."""

    def __init__(self, target: Model, draft, draft_layers: int, batch: int, K: int,
                 max_tokens: int, prompt_len: int, kv_bits=16, temperature=0.0, top_p=1.0,
                 seed=0, context_len=0, context_seed=0, seq_base=0, kv_quirk=0):
        self.cfg = SpecConfig(batch, K, max_tokens, prompt_len, kv_bits, temperature, top_p, seed,
                              context_len, context_seed, seq_base, kv_quirk)
        h = C.c_void_p()
        call("lmx_spec_create", target.h, draft.h if draft is not None else None, draft_layers,
             C.byref(self.cfg), C.byref(h))
        self.h = h
        self._keep = (target, draft)

    def prefill(self, prompts):
        import numpy as np
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        assert p.shape == (self.cfg.batch, self.cfg.prompt_len)
        call("lmx_spec_prefill", self.h, p.ctypes.data_as(C.c_void_p))

    def decode(self, use_graph=True):
        sec = C.c_double(0.0)
        call("lmx_spec_decode", self.h, 1 if use_graph else 0, C.byref(sec))
        return sec.value

    def result(self):
        import numpy as np
        out = np.zeros((self.cfg.batch, self.cfg.max_tokens), np.int32)
        st = np.zeros(5, np.int64)
        call("lmx_spec_result", self.h, out.ctypes.data_as(C.c_void_p),
             st.ctypes.data_as(C.c_void_p))
        return out, dict(steps=int(st[0]), proposed=int(st[1]), accepted=int(st[2]),
                         emitted=int(st[3]), replays=int(st[4]))

    def next(self):
        """TokenIterator::next(): the next token of every sequence (-1 once a
        sequence has produced max_tokens), or None when none is left."""
        import numpy as np
        out = np.zeros(self.cfg.batch, np.int32)
        live = C.c_int(0)
        call("lmx_spec_next", self.h, out.ctypes.data_as(C.c_void_p), C.byref(live))
        return out if live.value else None

    def generate(self, prompts, eos=(), should_cancel=None, on_token=None):
        """generate(): prefill, then tokens until every sequence stops (EOS,
        on_token returning True, max_tokens) or should_cancel() returns True.
        Returns the per-sequence CompletionInfo list."""
        import numpy as np
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        e = np.ascontiguousarray(list(eos), dtype=np.int32)
        cf = CANCEL_FN(lambda _u: 1 if should_cancel() else 0) if should_cancel else CANCEL_FN()
        tf = TOKEN_FN(lambda _u, b, t: 1 if on_token(b, t) else 0) if on_token else TOKEN_FN()
        info = (CompletionInfo * self.cfg.batch)()
        call("lmx_spec_generate", self.h, p.ctypes.data_as(C.c_void_p),
             e.ctypes.data_as(C.c_void_p) if e.size else None, int(e.size), cf, None, tf, None, info)
        return list(info)

    def profile(self, what, iters=20):
        sec, by = C.c_double(0.0), C.c_double(0.0)
        call("lmx_spec_profile", self.h, what, iters, C.byref(sec), C.byref(by))
        return sec.value, by.value

    def step_launches(self):
        n = C.c_int64(0)
        call("lmx_spec_step_launches", self.h, C.byref(n))
        return n.value

    def close(self):
        if self.h:
            lib().lmx_spec_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def lib():
    """Load liblmx.so (raises LmxError if the CUDA extension is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LmxError(f"CUDA extension missing: {LIB_PATH} (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc, what="lmx call"):
    if rc != 0:
        msg = lib().lmx_last_error().decode(errors="replace")
        raise LmxError(f"{what} failed with status {rc}: {msg}")
    return rc


def call(name, *args):
    return check(getattr(lib(), name)(*args), name)
