"""ctypes binding of libengine_cuda.so (include/engine_cuda.h, ec_transformer.h).

Used by tests/, bench.py and __graft_entry__.smoke().  The library is loaded
from this directory; there is no fallback: if it is missing or has no CUDA
device, calls raise.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libengine_cuda.so")

EC_OK, EC_ERR_ARG, EC_ERR_CUDA, EC_ERR_OOM, EC_ERR_STATE = 0, -1, -2, -3, -4
EC_ERR_UNSUPPORTED, EC_ERR_TIMEOUT = -5, -6
EC_W_INT8, EC_W_FP8, EC_W_BF16 = 0, 1, 2
EC_ATTN_REFERENCE, EC_ATTN_SPLIT = 0, 1
EC_WQ, EC_WK, EC_WV, EC_WO, EC_W1, EC_W2, EC_W3, EC_ATTN_NORM, EC_FFN_NORM = range(9)
EC_EMBEDDING, EC_FINAL_NORM, EC_LM_HEAD = 16, 17, 18
EC_FINAL_ADAPTER, EC_LOGIT_BIAS = 19, 20
MAT_IDS = {"wq": EC_WQ, "wk": EC_WK, "wv": EC_WV, "wo": EC_WO, "w1": EC_W1, "w2": EC_W2,
           "w3": EC_W3}

# every symbol include/*.h declares
EXPORTS = [
    "ec_last_error", "ec_config_default", "ec_create", "ec_destroy", "ec_set_weight",
    "ec_reset", "ec_decode_step", "ec_decode_step_device", "ec_logits_device",
    "ec_argmax_device", "ec_stream", "ec_synchronize", "ec_read_state", "ec_read_lsh",
    "ec_read_counters", "ec_launches_per_step", "ec_op_gemv", "ec_gemv_packed_bytes", "ec_gemv_pack",
    "ec_op_gemv_packed", "ec_op_gemv_packed_batch", "ec_op_rmsnorm", "ec_op_rope",
    "ec_op_silu_mul", "ec_op_quant_int8", "ec_op_argmax", "ec_op_paged_append",
    "ec_op_paged_attention", "ec_op_paged_attention_static", "ec_transformer_init", "ec_transformer_set_tensor",
    "ec_transformer_forward", "ec_transformer_argmax", "ec_transformer_reset",
    "ec_transformer_free", "ec_profile_enable", "ec_profile_read", "ec_lsh_attn_create",
    "ec_lsh_attn_destroy", "ec_lsh_attn_build", "ec_lsh_attn_query", "ec_lsh_attn_read",
    "ec_gemm_tc_bytes", "ec_gemm_tc_pack", "ec_op_gemm_tc", "ec_prefill", "ec_set_weight_bf16",
    "ec_tp_unique_id", "ec_create_tp", "ec_verify", "ec_lsh_attn_build_paged",
    "ec_op_sample_top_p", "ec_op_sample_temperature", "ec_set_context_bias",
]
K_NAMES = ["gemv_qkv", "gemv_o", "gemv_gateup", "gemv_down", "gemv_lm", "kv_append", "select",
           "attention", "embed", "argmax", "gemv_chain", "tc_gemm", "tc_quant", "tc_combine"]


class ModelConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "seq_len",
        "head_dim")] + [("rope_theta", C.c_float), ("norm_eps", C.c_float)] + [
        (n, C.c_int) for n in (
            "weight_kind", "use_paged_kv", "sparse_k", "window", "sparse_blocks_k",
            "lsh_tables", "lsh_bits", "lsh_unit", "lsh_max_units", "lsh_radius",
            "lsh_max_cand", "max_batch", "tensor_min_batch", "attention_mode", "wait_limit")]


class Transformer(C.Structure):
    _fields_ = [("config", ModelConfig), ("ctx", C.c_void_p), ("logits", C.POINTER(C.c_float)),
                ("last_token", C.c_int), ("last_error", C.c_int)]


class PagedView(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("k_scale", C.c_void_p),
                ("v_scale", C.c_void_p), ("centroid", C.c_void_p), ("page_table", C.c_void_p),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("max_blocks", C.c_int)]


class LshAttnConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_heads", "n_kv_heads", "head_dim", "max_tokens", "tables",
                                       "bits", "unit", "radius", "max_cand", "window", "top_k",
                                       "max_queries")]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run __graft_entry__.build()")
        L = C.CDLL(LIB_PATH)
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        sig = {
            "ec_last_error": (C.c_char_p, []),
            "ec_config_default": (i, [C.POINTER(ModelConfig)]),
            "ec_create": (i, [C.POINTER(ModelConfig), i, C.POINTER(vp)]),
            "ec_tp_unique_id": (i, [vp, C.c_size_t]),
            "ec_create_tp": (i, [C.POINTER(ModelConfig), i, i, i, vp, C.POINTER(vp)]),
            "ec_destroy": (None, [vp]),
            "ec_set_weight": (i, [vp, i, i, vp, vp, i]),
            "ec_set_weight_bf16": (i, [vp, i, i, vp, i]),
            "ec_reset": (i, [vp, i]),
            "ec_decode_step": (i, [vp, vp, vp, i, vp, vp]),
            "ec_decode_step_device": (i, [vp, vp, vp, i, i]),
            "ec_logits_device": (vp, [vp]),
            "ec_argmax_device": (vp, [vp]),
            "ec_stream": (vp, [vp]),
            "ec_synchronize": (i, [vp]),
            "ec_read_state": (i, [vp, i, i, vp, C.c_size_t]),
            "ec_read_lsh": (i, [vp, i, vp, vp, vp, vp, vp, vp]),
            "ec_read_counters": (i, [vp, i, vp]),
            "ec_launches_per_step": (i, [vp, i]),
            "ec_op_gemv": (i, [i, vp, vp, vp, vp, i, i, vp]),
            "ec_gemv_packed_bytes": (C.c_size_t, [i, i]),
            "ec_gemv_pack": (i, [vp, vp, i, i, vp]),
            "ec_gemm_tc_bytes": (C.c_size_t, [i, i]),
            "ec_gemm_tc_pack": (i, [vp, vp, i, i, vp]),
            "ec_op_gemm_tc": (i, [vp, vp, vp, vp, i, i, i, vp]),
            "ec_prefill": (i, [vp, i, vp, i, i, vp, vp]),
            "ec_verify": (i, [vp, i, vp, i, i, vp]),
            "ec_op_gemv_packed": (i, [i, vp, vp, vp, vp, i, i, vp]),
            "ec_op_gemv_packed_batch": (i, [i, vp, vp, vp, vp, i, i, i, vp]),
            "ec_op_rmsnorm": (i, [vp, vp, vp, i, f, vp]),
            "ec_op_rope": (i, [vp, i, i, i, vp, vp, i, vp]),
            "ec_op_silu_mul": (i, [vp, vp, vp, i, vp]),
            "ec_op_quant_int8": (i, [vp, vp, vp, i, i, vp]),
            "ec_op_argmax": (i, [vp, i, i, vp, vp]),
            "ec_op_sample_top_p": (i, [vp, i, i, vp, vp, i, f, f, f, i, vp, vp, vp]),
            "ec_op_sample_temperature": (i, [vp, i, i, f, vp, vp, vp]),
            "ec_set_context_bias": (i, [vp, vp, vp, vp, i]),
            "ec_op_paged_append": (i, [C.POINTER(PagedView), vp, vp, i, vp]),
            "ec_op_paged_attention": (i, [C.POINTER(PagedView), vp, vp, i, i, i, vp, vp, vp]),
            "ec_op_paged_attention_static": (i, [C.POINTER(PagedView), vp, vp, i, i, i, vp, vp,
                                                 vp]),
            "ec_transformer_init": (i, [C.POINTER(Transformer), C.POINTER(ModelConfig), i]),
            "ec_transformer_set_tensor": (i, [C.POINTER(Transformer), C.c_char_p, vp, vp]),
            "ec_transformer_forward": (C.POINTER(C.c_float), [C.POINTER(Transformer), i, i]),
            "ec_transformer_argmax": (i, [C.POINTER(Transformer)]),
            "ec_transformer_reset": (i, [C.POINTER(Transformer)]),
            "ec_transformer_free": (None, [C.POINTER(Transformer)]),
            "ec_lsh_attn_create": (i, [C.POINTER(LshAttnConfig), i, C.POINTER(vp)]),
            "ec_lsh_attn_destroy": (None, [vp]),
            "ec_lsh_attn_build": (i, [vp, vp, vp, i, vp]),
            "ec_lsh_attn_build_paged": (i, [vp, vp, vp, vp, i, vp]),
            "ec_lsh_attn_query": (i, [vp, vp, i, vp, vp, vp, vp]),
            "ec_lsh_attn_read": (i, [vp, i, vp, C.c_size_t]),
            "ec_profile_enable": (i, [vp, i]),
            "ec_profile_read": (i, [vp, i, C.POINTER(C.c_double), C.POINTER(i),
                                    C.POINTER(C.c_double)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class EngineError(RuntimeError):
    pass


def check(rc):
    if rc != EC_OK:
        raise EngineError(f"engine_cuda error {rc}: {lib().ec_last_error().decode()}")
    return rc


def config_from(cfg, weight_kind=EC_W_INT8, use_paged_kv=True, sparse_k=64, max_batch=1,
                **over):
    c = ModelConfig()
    check(lib().ec_config_default(C.byref(c)))
    for k in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
              "seq_len", "head_dim"):
        setattr(c, k, int(getattr(cfg, k)))
    c.rope_theta = float(cfg.rope_theta)
    c.norm_eps = float(cfg.norm_eps)
    c.weight_kind = weight_kind
    c.use_paged_kv = int(use_paged_kv)
    c.sparse_k = sparse_k
    c.max_batch = max_batch
    for k, v in over.items():
        setattr(c, k, v)
    return c


def _ptr(a):
    return C.c_void_p(a.ctypes.data) if a is not None else None


def tp_unique_id():
    """128 bytes naming a new tensor-parallel group (ec_tp_unique_id); one
    rank creates it, every rank passes the same bytes to Engine(tp=...)."""
    buf = C.create_string_buffer(128)
    check(lib().ec_tp_unique_id(buf, 128))
    return buf.raw


class Engine:
    """One decode context (ec_ctx) on one device.  tp=(rank, world, id):
    this rank of a tensor-parallel group (ec_create_tp)."""

    def __init__(self, cfg, device=0, tp=None, **kw):
        self.model_cfg = cfg
        self.c = config_from(cfg, **kw)
        self.h = C.c_void_p()
        if tp is None:
            check(lib().ec_create(C.byref(self.c), device, C.byref(self.h)))
        else:
            rank, world, uid = tp
            self._uid = C.create_string_buffer(bytes(uid), 128)
            check(lib().ec_create_tp(C.byref(self.c), device, rank, world, self._uid,
                                     C.byref(self.h)))

    def load(self, model):
        """Register a synth.Model (host numpy arrays)."""
        L = lib()
        for i, lw in enumerate(model.layers):
            for n, mid in MAT_IDS.items():
                q, s = lw[n]
                check(L.ec_set_weight(self.h, i, mid, _ptr(np.ascontiguousarray(q)),
                                      _ptr(np.ascontiguousarray(s)), 0))
            check(L.ec_set_weight(self.h, i, EC_ATTN_NORM, _ptr(lw["attention_norm"]), None, 0))
            check(L.ec_set_weight(self.h, i, EC_FFN_NORM, _ptr(lw["ffn_norm"]), None, 0))
        check(L.ec_set_weight(self.h, -1, EC_EMBEDDING, _ptr(model.emb), None, 0))
        check(L.ec_set_weight(self.h, -1, EC_FINAL_NORM, _ptr(model.final_norm), None, 0))
        check(L.ec_set_weight(self.h, -1, EC_LM_HEAD, _ptr(model.lm[0]), _ptr(model.lm[1]), 0))

    def load_bf16(self, bf):
        """Register BF16 host weights (synth.Model.bf16_weights() form); the
        matrices are quantised on the device (ec_set_weight_bf16)."""
        L = lib()
        for i, lw in enumerate(bf["layers"]):
            for n, mid in MAT_IDS.items():
                check(L.ec_set_weight_bf16(self.h, i, mid, _ptr(np.ascontiguousarray(lw[n])), 0))
            check(L.ec_set_weight(self.h, i, EC_ATTN_NORM, _ptr(lw["attention_norm"]), None, 0))
            check(L.ec_set_weight(self.h, i, EC_FFN_NORM, _ptr(lw["ffn_norm"]), None, 0))
        check(L.ec_set_weight(self.h, -1, EC_EMBEDDING, _ptr(bf["emb"]), None, 0))
        check(L.ec_set_weight(self.h, -1, EC_FINAL_NORM, _ptr(bf["final_norm"]), None, 0))
        check(L.ec_set_weight_bf16(self.h, -1, EC_LM_HEAD, _ptr(bf["lm"]), 0))

    def set_final(self, adapter=None, logit_bias=None):
        """Register the optional final hidden adapter (bf16 [dim][dim] host
        array) and logit bias (float [vocab]); an all-zero tensor stays off."""
        L = lib()
        if adapter is not None:
            check(L.ec_set_weight(self.h, -1, EC_FINAL_ADAPTER,
                                  _ptr(np.ascontiguousarray(adapter, np.uint16)), None, 0))
        if logit_bias is not None:
            check(L.ec_set_weight(self.h, -1, EC_LOGIT_BIAS,
                                  _ptr(np.ascontiguousarray(logit_bias, np.float32)), None, 0))

    def set_context_bias(self, keys, tokens, biases):
        """The reference's context-aware bias cache (t_transformer.context_bias):
        uint64 keys (0 = empty), int32 target tokens, float biases."""
        keys = np.ascontiguousarray(keys, np.uint64)
        tokens = np.ascontiguousarray(tokens, np.int32)
        biases = np.ascontiguousarray(biases, np.float32)
        check(lib().ec_set_context_bias(self.h, _ptr(keys), _ptr(tokens), _ptr(biases),
                                        keys.size))

    def set_weight_device(self, layer, which, ptr, scale_ptr):
        check(lib().ec_set_weight(self.h, layer, which, C.c_void_p(ptr),
                                  C.c_void_p(scale_ptr) if scale_ptr else None, 1))

    def reset(self, seq=0):
        check(lib().ec_reset(self.h, seq))

    def step(self, tokens, pos, want_logits=True, out=None):
        """One decode step through ec_decode_step with host buffers.  `out`
        (optional): caller-owned (logits [B][vocab] float32, argmax [B] int32)
        arrays to fill instead of new ones -- e.g. views of pinned memory, as
        a serving loop keeps them."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        B = tokens.size
        if out is not None:
            lg, am = out
            lg = lg if want_logits else None
        else:
            lg = np.empty((B, self.c.vocab_size), np.float32) if want_logits else None
            am = np.empty(B, np.int32)
        check(lib().ec_decode_step(self.h, _ptr(tokens), _ptr(pos), B, _ptr(lg), _ptr(am)))
        return lg, am

    def state(self, which, seq=0, n=None):
        n = n or max(self.c.vocab_size, self.c.hidden_dim, self.c.n_heads * self.c.head_dim)
        out = np.zeros(n, np.float32)
        check(lib().ec_read_state(self.h, which, seq, _ptr(out), n))
        return out

    def lsh(self, seq=0):
        c = self.c
        mu = c.lsh_max_units
        n = C.c_int()
        uh = np.zeros(c.lsh_tables * mu, np.uint32)
        us = np.zeros(mu, np.int32)
        ul = np.zeros(mu, np.int32)
        hd = np.zeros(c.lsh_tables << c.lsh_bits, np.int32)
        nx = np.zeros(c.lsh_tables * mu, np.int32)
        check(lib().ec_read_lsh(self.h, seq, C.byref(n), _ptr(uh), _ptr(us), _ptr(ul), _ptr(hd),
                                _ptr(nx)))
        return dict(n_units=n.value, unit_hash=uh.reshape(c.lsh_tables, mu), unit_start=us,
                    unit_len=ul, heads=hd.reshape(c.lsh_tables, -1),
                    next=nx.reshape(c.lsh_tables, mu))

    def counters(self, seq=0):
        out = np.zeros(2, np.uint64)
        check(lib().ec_read_counters(self.h, seq, _ptr(out)))
        return int(out[0]), int(out[1])

    def profile(self, on):
        check(lib().ec_profile_enable(self.h, int(on)))

    def profile_read(self):
        out = {}
        for k, name in enumerate(K_NAMES):
            ms, n, by = C.c_double(), C.c_int(), C.c_double()
            check(lib().ec_profile_read(self.h, k, C.byref(ms), C.byref(n), C.byref(by)))
            out[name] = dict(ms=ms.value, launches=n.value, bytes=by.value)
        return out

    def prefill(self, seq, tokens, pos0=0):
        """Tokens of one sequence as rows of batched steps; returns the last
        token's logits and greedy token."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        lg = np.empty(self.c.vocab_size, np.float32)
        am = np.empty(1, np.int32)
        check(lib().ec_prefill(self.h, int(seq), _ptr(tokens), tokens.size, int(pos0), _ptr(lg),
                               _ptr(am)))
        return lg, int(am[0])

    def verify(self, seq, tokens, pos0):
        """Greedy token after each of `tokens` (ec_verify)."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(tokens.size, np.int32)
        check(lib().ec_verify(self.h, int(seq), _ptr(tokens), tokens.size, int(pos0), _ptr(out)))
        return out

    def sample_device(self, B, r_ptr, out_ptr, history_ptr=None, history_len_ptr=None,
                      history_stride=0, temperature=0.7, top_p=0.9, penalty=1.2,
                      block_token0=True):
        """The server's sampling step (worker.c:436-497) on the last step's
        device logits, on the context's stream: no logits leave the device.
        out_ptr may be the next step's tokens_dev."""
        check(lib().ec_op_sample_top_p(
            lib().ec_logits_device(self.h), self.c.vocab_size, B,
            C.c_void_p(history_ptr) if history_ptr else None,
            C.c_void_p(history_len_ptr) if history_len_ptr else None, int(history_stride),
            float(temperature), float(top_p), float(penalty), int(block_token0),
            C.c_void_p(r_ptr), C.c_void_p(out_ptr), self.stream()))

    def step_device(self, tokens_ptr, pos_ptr, B, feedback=True):
        check(lib().ec_decode_step_device(self.h, C.c_void_p(tokens_ptr), C.c_void_p(pos_ptr),
                                          B, int(feedback)))

    def sync(self):
        check(lib().ec_synchronize(self.h))

    def stream(self):
        return lib().ec_stream(self.h)

    def launches_per_step(self, B=1):
        return lib().ec_launches_per_step(self.h, B)

    def close(self):
        if self.h:
            lib().ec_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def speculate(target, draft, token, pos, n_draft, seq=0):
    """One burst of mtp_generate (speculate.c:93-258) with two engines of one
    vocabulary: the draft decodes n_draft greedy tokens from `token` at
    `pos`, the target verifies them in one ec_verify pass; returns the
    target's tokens for the accepted prefix plus its correction (at most
    n_draft tokens), exactly the greedy tokens the target alone would give.
    Both engines' caches stay valid for the returned tokens (positions past
    them are overwritten by the next steps)."""
    drafts, cur = [], int(token)
    for i in range(n_draft):
        _, am = draft.step([cur], [pos + i], want_logits=False)
        cur = int(am[0])
        drafts.append(cur)
    checks = [int(token)] + drafts[:-1]
    pred = target.verify(seq, checks, pos)
    out = []
    for i in range(n_draft):
        out.append(int(pred[i]))
        if int(pred[i]) != drafts[i]:
            break
    return out


class HostTransformer:
    """The reference-facing API: ec_transformer_init / _forward (host logits)."""

    def __init__(self, cfg, device=0, **kw):
        self.t = Transformer()
        self.c = config_from(cfg, **kw)
        check(lib().ec_transformer_init(C.byref(self.t), C.byref(self.c), device))
        self.vocab = cfg.vocab_size

    def load(self, model):
        """Register tensors by the reference's HuggingFace names."""
        hf = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj",
              "wo": "self_attn.o_proj", "w1": "mlp.gate_proj", "w2": "mlp.down_proj",
              "w3": "mlp.up_proj"}
        L = lib()
        for i, lw in enumerate(model.layers):
            for n, hn in hf.items():
                q, s = lw[n]
                check(L.ec_transformer_set_tensor(
                    C.byref(self.t), f"model.layers.{i}.{hn}.weight".encode(), _ptr(q), _ptr(s)))
            check(L.ec_transformer_set_tensor(C.byref(self.t),
                  f"model.layers.{i}.input_layernorm.weight".encode(),
                  _ptr(lw["attention_norm"]), None))
            check(L.ec_transformer_set_tensor(C.byref(self.t),
                  f"model.layers.{i}.post_attention_layernorm.weight".encode(),
                  _ptr(lw["ffn_norm"]), None))
        check(L.ec_transformer_set_tensor(C.byref(self.t), b"model.embed_tokens.weight",
                                          _ptr(model.emb), None))
        check(L.ec_transformer_set_tensor(C.byref(self.t), b"model.norm.weight",
                                          _ptr(model.final_norm), None))
        check(L.ec_transformer_set_tensor(C.byref(self.t), b"lm_head.weight",
                                          _ptr(model.lm[0]), _ptr(model.lm[1])))

    def forward(self, token, pos):
        p = lib().ec_transformer_forward(C.byref(self.t), int(token), int(pos))
        if not p:
            check(self.t.last_error or EC_ERR_STATE)
        return np.ctypeslib.as_array(p, (self.vocab,))

    def argmax(self):
        return lib().ec_transformer_argmax(C.byref(self.t))

    def close(self):
        if self.t.ctx:
            lib().ec_transformer_free(C.byref(self.t))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
