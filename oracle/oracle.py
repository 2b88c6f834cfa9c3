"""Oracle bindings -- TEST INFRASTRUCTURE ONLY.

ctypes access to
  * ``libec_port.so``            -- this repository's C restatement (oracle/port),
  * ``_ref/libref_driver.so``    -- the reference engine's own sources compiled
                                    in place (oracle/Makefile, target ``ref``).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module, and only as the checker / the CPU baseline.  The product
(libengine_cuda.so) never loads either library.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "libec_port.so")
REF_SO = os.path.join(HERE, "_ref", "libref_driver.so")
DROPIN_SO = os.path.join(HERE, "_ref", "libref_dropin.so")

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


def _sig(lib, name, res, *args):
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = list(args)
    return fn


class PortConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
        "seq_len", "head_dim")] + [("rope_theta", C.c_float), ("norm_eps", C.c_float)] + [
        (n, C.c_int) for n in (
            "use_paged_kv", "sparse_k", "window", "sparse_blocks_k", "lsh_tables",
            "lsh_bits", "lsh_unit", "lsh_max_units", "lsh_radius", "lsh_max_cand",
            "weight_kind")]


class PortWeights(C.Structure):
    _fields_ = [("emb", C.c_void_p), ("final_norm", C.c_void_p), ("lm", C.c_void_p),
                ("lm_scale", C.c_void_p), ("mat", C.POINTER(C.c_void_p)),
                ("mat_scale", C.POINTER(C.c_void_p)), ("norm", C.POINTER(C.c_void_p))]


class RefdConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
        "seq_len", "head_dim")] + [("rope_theta", C.c_float), ("norm_eps", C.c_float),
                                   ("use_paged_kv", C.c_int), ("sparse_k", C.c_int)]


class LshIndex(C.Structure):
    """Mirror of t_lsh_index (src/compute/ops_lsh.h:70-85) for introspection."""
    _fields_ = [("block_hashes", C.c_uint16 * 4096), ("block_starts", C.c_int * 4096),
                ("block_lens", C.c_int * 4096), ("n_blocks", C.c_int),
                ("bucket_heads", C.c_int * 65536), ("chain_next", C.c_int * 4096),
                ("sum_buffer", C.c_float * 256), ("count", C.c_int), ("start_pos", C.c_int),
                ("block_size", C.c_int)]


class PortLsh(C.Structure):
    _fields_ = [("n_tables", C.c_int), ("n_bits", C.c_int), ("dim", C.c_int),
                ("unit", C.c_int), ("max_units", C.c_int), ("radius", C.c_int),
                ("hp", C.POINTER(C.c_float)), ("unit_hash", C.POINTER(C.c_uint32)),
                ("unit_start", C.POINTER(C.c_int)), ("unit_len", C.POINTER(C.c_int)),
                ("heads", C.POINTER(C.c_int)), ("next", C.POINTER(C.c_int)),
                ("n_units", C.c_int), ("acc", C.POINTER(C.c_float)),
                ("acc_count", C.c_int), ("acc_start", C.c_int)]


class PortPaged(C.Structure):
    _fields_ = [("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("max_blocks", C.c_int),
                ("n_blocks", C.c_int), ("n_tokens", C.c_int),
                ("k", C.POINTER(C.c_int8)), ("v", C.POINTER(C.c_int8)),
                ("ks", C.POINTER(C.c_float)), ("vs", C.POINTER(C.c_float)),
                ("centroid", C.POINTER(C.c_float)), ("fill", C.POINTER(C.c_int))]


_port = None
_ref = None


def port():
    """The C restatement (always buildable)."""
    global _port
    if _port is None:
        lib = C.CDLL(PORT_SO)
        _sig(lib, "port_gemv_bf16", None, f32p, u16p, f32p, C.c_int, C.c_int)
        _sig(lib, "port_gemv_q8", None, f32p, i8p, f32p, f32p, C.c_int, C.c_int)
        _sig(lib, "port_gemv_fp8", None, f32p, u8p, C.c_float, f32p, C.c_int, C.c_int)
        _sig(lib, "port_rmsnorm", None, f32p, f32p, u16p, C.c_int, C.c_float)
        _sig(lib, "port_rope_tables", None, f32p, f32p, C.c_int, C.c_int, C.c_float)
        _sig(lib, "port_rope", None, f32p, C.c_int, C.c_int, C.c_int, f32p, f32p, C.c_int)
        _sig(lib, "port_silu_mul", None, f32p, f32p, f32p, C.c_int)
        _sig(lib, "port_quant_int8", C.c_float, i8p, f32p, C.c_int)
        _sig(lib, "port_argmax", C.c_int, f32p, C.c_int)
        _sig(lib, "port_sample_top_p", C.c_int, f32p, C.c_int, i32p, C.c_int, C.c_float,
             C.c_float, C.c_float, C.c_int, C.c_float, i32p, f32p)
        _sig(lib, "port_sample_temperature", C.c_int, f32p, C.c_int, C.c_float, C.c_float)
        _sig(lib, "port_heap_topk", C.c_int, f32p, i32p, C.c_int, C.c_int, i32p)
        _sig(lib, "port_fast_expf", C.c_float, C.c_float)
        _sig(lib, "port_fast_expf_vec", C.c_float, C.c_float)
        _sig(lib, "port_fp8_e4m3_to_f32", C.c_float, C.c_uint8)
        _sig(lib, "port_dot_f32", C.c_float, f32p, f32p, C.c_int)
        _sig(lib, "port_dot_bf16_f32", C.c_float, u16p, f32p, C.c_int)
        _sig(lib, "port_lsh_create", C.POINTER(PortLsh), C.c_int, C.c_int, C.c_int, C.c_int,
             C.c_int, C.c_int, C.c_uint)
        _sig(lib, "port_lsh_free", None, C.POINTER(PortLsh))
        _sig(lib, "port_lsh_hash", C.c_uint32, C.POINTER(PortLsh), C.c_int, f32p)
        _sig(lib, "port_lsh_update", None, C.POINTER(PortLsh), f32p, C.c_int)
        _sig(lib, "port_lsh_find", C.c_int, C.POINTER(PortLsh),
             np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS"), i32p, C.c_int)
        _sig(lib, "port_lsh_attend", C.c_int, C.POINTER(PortLsh), u16p, u16p, C.c_int, f32p,
             C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, i32p, f32p)
        _sig(lib, "port_paged_create", C.POINTER(PortPaged), C.c_int, C.c_int, C.c_int)
        _sig(lib, "port_paged_free", None, C.POINTER(PortPaged))
        _sig(lib, "port_paged_append", None, C.POINTER(PortPaged), f32p, f32p, C.c_int)
        _sig(lib, "port_paged_attention", None, f32p, f32p, C.POINTER(PortPaged), i32p,
             C.c_int, C.c_int)
        _sig(lib, "port_paged_scores", None, C.POINTER(PortPaged), f32p, f32p)
        _sig(lib, "port_select_blocks", C.c_int, f32p, C.c_int, C.c_int, i32p)
        _sig(lib, "port_linear_attention", None, f32p, f32p, u16p, u16p, i32p, C.c_int,
             C.c_int, C.c_int, C.c_int)
        _sig(lib, "port_model_create", C.c_void_p, C.POINTER(PortConfig),
             C.POINTER(PortWeights))
        _sig(lib, "port_model_free", None, C.c_void_p)
        _sig(lib, "port_model_reset", None, C.c_void_p)
        _sig(lib, "port_model_forward", C.POINTER(C.c_float), C.c_void_p, C.c_int, C.c_int)
        _sig(lib, "port_model_state", C.POINTER(C.c_float), C.c_void_p, C.c_int)
        _sig(lib, "port_model_lsh", C.POINTER(PortLsh), C.c_void_p)
        _sig(lib, "port_model_paged", C.POINTER(PortPaged), C.c_void_p, C.c_int)
        _sig(lib, "port_model_linear_k", C.POINTER(C.c_uint16), C.c_void_p, C.c_int)
        _sig(lib, "port_model_counters", None, C.c_void_p, C.POINTER(C.c_ulonglong))
        _port = lib
    return _port


def ref_available():
    return os.path.exists(REF_SO)


def dropin_available():
    return os.path.exists(DROPIN_SO)


_dropin = None


def dropin():
    """The reference engine built with the drop-in hook (oracle/dropin.py):
    its transformer_forward calls libengine_cuda.so once a context is
    attached with refd_attach_gpu.  Load libengine_cuda.so first (the engine
    binding) so that both share one copy of it."""
    global _dropin
    if _dropin is None:
        _dropin = _bind(C.CDLL(DROPIN_SO))
        _sig(_dropin, "refd_attach_gpu", None, C.c_void_p, C.c_void_p)
    return _dropin


def ref():
    """The reference engine's own code, compiled from its sources by oracle/Makefile."""
    global _ref
    if _ref is None:
        _ref = _bind(C.CDLL(REF_SO))
    return _ref


def _bind(lib):
    """Signatures of the refd_* driver calls (ref_driver.c)."""
    vp = C.c_void_p
    _sig(lib, "refd_create", vp, C.POINTER(RefdConfig), vp, vp, vp, C.POINTER(vp))
    _sig(lib, "refd_forward", C.POINTER(C.c_float), vp, C.c_int, C.c_int)
    _sig(lib, "refd_fill_context", C.c_int, vp, C.c_int, C.c_uint)
    _sig(lib, "refd_set_adapter", None, vp, vp)
    _sig(lib, "refd_set_logit_bias", None, vp, vp)
    _sig(lib, "refd_state", C.POINTER(C.c_float), vp, C.c_int)
    _sig(lib, "refd_lsh_index", C.POINTER(LshIndex), vp)
    _sig(lib, "refd_paged_block", C.c_int, vp, C.c_int, C.c_int, i8p, i8p, f32p, f32p,
         f32p)
    _sig(lib, "refd_linear_k", C.POINTER(C.c_uint16), vp, C.c_int)
    _sig(lib, "refd_lsh_counters", None, vp, C.POINTER(C.c_ulonglong))
    _sig(lib, "refd_matmul", C.c_int, f32p, u16p, f32p, C.c_int, C.c_int)
    _sig(lib, "refd_rmsnorm", None, f32p, f32p, u16p, C.c_int, C.c_float)
    _sig(lib, "refd_rope_create", vp, C.c_int, C.c_int, C.c_float)
    _sig(lib, "refd_rope_table", C.POINTER(C.c_float), vp, C.c_int)
    _sig(lib, "refd_rope_apply", None, vp, f32p, C.c_int, C.c_int)
    _sig(lib, "refd_silu_mul", None, f32p, f32p, f32p, C.c_int)
    _sig(lib, "refd_quant_int8", C.c_float, i8p, f32p, C.c_int)
    _sig(lib, "refd_argmax", C.c_int, f32p, C.c_int)
    _sig(lib, "refd_first_rand", C.c_float, C.c_uint)
    _sig(lib, "refd_set_context_bias", None, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
         C.c_int)
    _sig(lib, "refd_sample_top_p", C.c_int, f32p, C.c_int, C.c_float, C.c_float, C.c_uint)
    _sig(lib, "refd_heap_topk", C.c_int, f32p, i32p, C.c_int, C.c_int, i32p)
    _sig(lib, "refd_lsh_ctx_create", vp, C.c_int, C.c_uint)
    _sig(lib, "refd_lsh_hyperplanes", C.POINTER(C.c_float), vp)
    _sig(lib, "refd_lsh_hash", C.c_int, vp, f32p)
    _sig(lib, "refd_lsh_index_create", vp)
    _sig(lib, "refd_lsh_update", None, vp, vp, f32p, C.c_int, C.c_int)
    _sig(lib, "refd_lsh_find", C.c_int, vp, C.c_int, i32p, C.c_int)
    _sig(lib, "refd_paged_create", vp, C.c_int, C.c_int, C.c_int)
    _sig(lib, "refd_paged_append", None, vp, f32p, f32p, C.c_int)
    _sig(lib, "refd_paged_phys", C.c_int, vp, C.c_int)
    _sig(lib, "refd_paged_nblocks", C.c_int, vp)
    _sig(lib, "refd_paged_attention", None, vp, f32p, f32p, C.c_int, C.c_int, C.c_int)
    _sig(lib, "refd_paged_sparse", C.c_int, vp, f32p, f32p, C.c_int, C.c_int, C.c_int,
         C.c_int, i32p)
    _sig(lib, "refd_paged_scores", None, vp, f32p, f32p)
    _sig(lib, "refd_linear_sparse_attention", None, f32p, f32p, u16p, u16p, C.c_int,
         i32p, C.c_int, C.c_int, C.c_int, C.c_int)
    return lib


# ---------------------------------------------------------------------------
# model wrappers
# ---------------------------------------------------------------------------
REF_DEFAULTS = dict(window=128, sparse_blocks_k=64, lsh_tables=1, lsh_bits=16, lsh_unit=64,
                    lsh_max_units=4096, lsh_radius=4, lsh_max_cand=64)


class PortModel:
    """The restated decode step over a synthetic model (see synth.py)."""

    def __init__(self, model, use_paged_kv=True, sparse_k=64, **lsh):
        cfg = model.cfg
        opts = dict(REF_DEFAULTS)
        opts.update(lsh)
        self._keep = []
        c = PortConfig(dim=cfg.dim, hidden_dim=cfg.hidden_dim, n_layers=cfg.n_layers,
                       n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
                       vocab_size=cfg.vocab_size, seq_len=cfg.seq_len, head_dim=cfg.head_dim,
                       rope_theta=cfg.rope_theta, norm_eps=cfg.norm_eps,
                       use_paged_kv=int(use_paged_kv), sparse_k=sparse_k,
                       weight_kind=0 if model.kind == "int8" else 1, **opts)
        L = cfg.n_layers
        mats = (C.c_void_p * (L * 7))()
        scs = (C.c_void_p * (L * 7))()
        norms = (C.c_void_p * (L * 2))()
        names = ("wq", "wk", "wv", "wo", "w1", "w2", "w3")
        for i in range(L):
            for j, n in enumerate(names):
                q, s = model.layers[i][n]
                mats[i * 7 + j] = q.ctypes.data
                scs[i * 7 + j] = s.ctypes.data
            norms[i * 2] = model.layers[i]["attention_norm"].ctypes.data
            norms[i * 2 + 1] = model.layers[i]["ffn_norm"].ctypes.data
        w = PortWeights(emb=model.emb.ctypes.data, final_norm=model.final_norm.ctypes.data,
                        lm=model.lm[0].ctypes.data, lm_scale=model.lm[1].ctypes.data,
                        mat=mats, mat_scale=scs, norm=norms)
        self._keep += [mats, scs, norms, w, c, model]
        self.cfg = cfg
        self.lib = port()
        self.h = self.lib.port_model_create(C.byref(c), C.byref(w))

    def forward(self, token, pos):
        p = self.lib.port_model_forward(self.h, token, pos)
        return np.ctypeslib.as_array(p, (self.cfg.vocab_size,)).copy()

    def reset(self):
        self.lib.port_model_reset(self.h)

    def counters(self):
        out = (C.c_ulonglong * 2)()
        self.lib.port_model_counters(self.h, out)
        return int(out[0]), int(out[1])

    def lsh(self):
        return self.lib.port_model_lsh(self.h).contents

    def paged(self, layer):
        return self.lib.port_model_paged(self.h, layer).contents

    def __del__(self):
        try:
            self.lib.port_model_free(self.h)
        except Exception:
            pass


class RefModel:
    """transformer_forward of the reference over BF16 weights W = q * scale.

    With power-of-two INT8 scales (synth.make_model(pow2=True)) those weights
    are exactly the INT8 model's weights, so its logits must match the CUDA
    path's bit for bit.
    """

    def __init__(self, model, use_paged_kv=True, sparse_k=64, lib=None):
        cfg = model.cfg
        self.cfg = cfg
        bf = model.bf16_weights()
        self._keep = [bf]
        L = cfg.n_layers
        ptrs = (C.c_void_p * (L * 9))()
        for i in range(L):
            lw = bf["layers"][i]
            for j, n in enumerate(("wq", "wk", "wv", "wo", "w1", "w2", "w3",
                                   "attention_norm", "ffn_norm")):
                ptrs[i * 9 + j] = lw[n].ctypes.data
        c = RefdConfig(dim=cfg.dim, hidden_dim=cfg.hidden_dim, n_layers=L, n_heads=cfg.n_heads,
                       n_kv_heads=cfg.n_kv_heads, vocab_size=cfg.vocab_size,
                       seq_len=cfg.seq_len, head_dim=cfg.head_dim, rope_theta=cfg.rope_theta,
                       norm_eps=cfg.norm_eps, use_paged_kv=int(use_paged_kv),
                       sparse_k=sparse_k)
        self._keep += [ptrs, c]
        self.lib = lib or ref()
        self.h = self.lib.refd_create(C.byref(c), bf["emb"].ctypes.data,
                                      bf["final_norm"].ctypes.data, bf["lm"].ctypes.data, ptrs)

    def forward(self, token, pos):
        p = self.lib.refd_forward(self.h, token, pos)
        return np.ctypeslib.as_array(p, (self.cfg.vocab_size,)).copy()

    def counters(self):
        out = (C.c_ulonglong * 2)()
        self.lib.refd_lsh_counters(self.h, out)
        return int(out[0]), int(out[1])

    def set_final(self, adapter=None, logit_bias=None):
        """Attach the final hidden adapter (bf16 [dim][dim]) and the logit bias
        (float [vocab]); None detaches."""
        self._keep += [adapter, logit_bias]
        self.lib.refd_set_adapter(self.h, adapter.ctypes.data if adapter is not None else None)
        self.lib.refd_set_logit_bias(self.h,
                                     logit_bias.ctypes.data if logit_bias is not None else None)

    def set_context_bias(self, keys=None, tokens=None, biases=None):
        """Attach the context-aware bias cache (uint64 keys, int32 target
        tokens, float biases, one table size); None detaches."""
        if keys is None:
            self.lib.refd_set_context_bias(self.h, None, None, None, 0)
            return
        keys = np.ascontiguousarray(keys, np.uint64)
        tokens = np.ascontiguousarray(tokens, np.int32)
        biases = np.ascontiguousarray(biases, np.float32)
        self._keep += [keys, tokens, biases]
        self.lib.refd_set_context_bias(self.h, keys.ctypes.data, tokens.ctypes.data,
                                       biases.ctypes.data, int(keys.size))

    def fill_context(self, n, seed=1):
        """Positions 0..n-1 of the paged cache from synthetic K/V through the
        reference's paged_kv_append and lsh_update (no projections)."""
        if self.lib.refd_fill_context(self.h, int(n), int(seed)) != 0:
            raise RuntimeError("refd_fill_context failed")

    def lsh_index(self):
        return self.lib.refd_lsh_index(self.h).contents
