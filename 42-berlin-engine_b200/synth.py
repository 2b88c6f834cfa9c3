"""Seeded synthetic Llama-style decoders for tests and the benchmark.

The reference ships no weights (its benches need Ministral/SmolLM checkpoints
that are not in the repository), so every run here uses random-init models of
the configured shapes, the same approach as the reference's
scripts/gen_dummy.py:18-48:

* matrices ~ N(0, 0.02), quantised per output row to symmetric INT8 with an
  fp32 scale (``pow2=True`` rounds each scale up to a power of two, which makes
  q * scale exactly representable in BF16, so the reference's BF16 path sees
  the identical weights), or cast to FP8 E4M3 with one per-tensor scale;
* token embedding BF16 ~ N(0, 0.02); RMSNorm weights BF16 1 + N(0, 0.1).
"""
from dataclasses import dataclass, asdict

import numpy as np


@dataclass
class ModelConfig:
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    seq_len: int
    head_dim: int
    rope_theta: float
    norm_eps: float = 1e-5

    def as_dict(self):
        return asdict(self)


TINY = ModelConfig(dim=512, hidden_dim=1408, n_layers=8, n_heads=8, n_kv_heads=8,
                   vocab_size=32000, seq_len=8192, head_dim=64, rope_theta=1e4)
LLAMA3_8B = ModelConfig(dim=4096, hidden_dim=14336, n_layers=32, n_heads=32, n_kv_heads=8,
                        vocab_size=128256, seq_len=8192, head_dim=128, rope_theta=5e5)
LLAMA_70B = ModelConfig(dim=8192, hidden_dim=28672, n_layers=80, n_heads=64, n_kv_heads=8,
                        vocab_size=128256, seq_len=32768, head_dim=128, rope_theta=5e5)

MATS = ("wq", "wk", "wv", "wo", "w1", "w2", "w3")


def mat_shapes(cfg):
    qd = cfg.n_heads * cfg.head_dim
    kvd = cfg.n_kv_heads * cfg.head_dim
    return {"wq": (qd, cfg.dim), "wk": (kvd, cfg.dim), "wv": (kvd, cfg.dim),
            "wo": (cfg.dim, qd), "w1": (cfg.hidden_dim, cfg.dim),
            "w2": (cfg.dim, cfg.hidden_dim), "w3": (cfg.hidden_dim, cfg.dim)}


def f32_to_bf16(a):
    """Round-to-nearest-even, as src/tensor/tensor.c:67-76 does."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(a):
    return (a.astype(np.uint32) << 16).view(np.float32)


def quant_int8_rows(w, pow2=True):
    amax = np.abs(w).max(axis=1)
    amax = np.where(amax > 0, amax, 1.0).astype(np.float32)
    if pow2:
        s = np.exp2(np.ceil(np.log2(amax / np.float32(127.0)))).astype(np.float32)
    else:
        s = (amax / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s


_E4M3 = None


def e4m3_table():
    """Decode value of every E4M3 code as the reference defines it
    (src/compute/ops_quant.c:27-50; no NaN code)."""
    global _E4M3
    if _E4M3 is None:
        t = np.zeros(256, np.float32)
        for c in range(256):
            e, m = (c >> 3) & 15, c & 7
            v = np.ldexp(m / 8.0, -6) if e == 0 else np.ldexp(1.0 + m / 8.0, e - 7)
            t[c] = -v if c & 0x80 else v
        _E4M3 = t
    return _E4M3


def quant_fp8_tensor(w):
    """Per-tensor E4M3 with a power-of-two scale; round to the nearest code
    (ties to even mantissa) among codes 0x00..0x7E (the OCP E4M3 cast; the
    NaN code 0x7F is never produced)."""
    amax = float(np.abs(w).max()) or 1.0
    s = np.float32(2.0 ** np.ceil(np.log2(amax / 448.0)))
    x = (w / s).astype(np.float32)
    pos = e4m3_table()[:0x7F]          # ascending magnitudes 0 .. 448
    a = np.abs(x)
    i = np.clip(np.searchsorted(pos, a), 1, 0x7E)
    lo, hi = pos[i - 1], pos[i]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & ((i & 1) == 0))
    code = np.where(pick_hi, i, i - 1).astype(np.uint8)
    code = np.where(x < 0, code | 0x80, code).astype(np.uint8)
    code = np.where(code == 0x80, 0, code).astype(np.uint8)
    return code, np.array([s], np.float32)


class Model:
    """Host copy of a synthetic model: quantised matrices + BF16 vectors."""

    def __init__(self, cfg, kind, emb, final_norm, lm, layers, seed):
        self.cfg, self.kind, self.emb, self.final_norm = cfg, kind, emb, final_norm
        self.lm, self.layers, self.seed = lm, layers, seed

    def dequant(self, q, s):
        if self.kind == "int8":
            return q.astype(np.float32) * s[:, None]
        return e4m3_table()[q] * s[0]

    def bf16_weights(self):
        """BF16 matrices q * scale for the reference's BF16 path."""
        out = {"emb": self.emb, "final_norm": self.final_norm,
               "lm": f32_to_bf16(self.dequant(*self.lm)), "layers": []}
        for lw in self.layers:
            d = {n: f32_to_bf16(self.dequant(*lw[n])) for n in MATS}
            d["attention_norm"] = lw["attention_norm"]
            d["ffn_norm"] = lw["ffn_norm"]
            out["layers"].append(d)
        return out


def make_model(cfg, seed=1234, kind="int8", pow2=True):
    rng = np.random.default_rng(seed)
    shapes = mat_shapes(cfg)

    def mat(shape):
        w = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
        return quant_int8_rows(w, pow2) if kind == "int8" else quant_fp8_tensor(w)

    def norm():
        return f32_to_bf16(1.0 + 0.1 * rng.standard_normal(cfg.dim, dtype=np.float32))

    emb = f32_to_bf16(rng.standard_normal((cfg.vocab_size, cfg.dim), dtype=np.float32)
                      * np.float32(0.02))
    layers = []
    for _ in range(cfg.n_layers):
        lw = {n: mat(shapes[n]) for n in MATS}
        lw["attention_norm"] = norm()
        lw["ffn_norm"] = norm()
        layers.append(lw)
    final_norm = norm()
    lm = mat((cfg.vocab_size, cfg.dim))
    return Model(cfg, kind, emb, final_norm, lm, layers, seed)


def prompt(cfg, n, seed=99):
    return np.random.default_rng(seed).integers(0, cfg.vocab_size, n).astype(np.int32)


class DeviceModel:
    """A synthetic model generated on a CUDA device with torch (same
    distributions as make_model), for shapes too large to generate on the
    host quickly.  torch is used for device memory only."""

    def __init__(self, cfg, seed=1234, device=0, kind="int8"):
        import torch
        self.cfg, self.kind, self.seed = cfg, kind, seed
        self.dev = torch.device("cuda", device)
        self.torch = torch
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)
        self._g = g

    def _normal(self, shape, scale):
        t = self.torch.randn(shape, generator=self._g, device=self.dev, dtype=self.torch.float32)
        return t.mul_(scale)

    def quant(self, w):
        """INT8 per row with power-of-two scales (as quant_int8_rows), or FP8
        E4M3 with one power-of-two scale per tensor (as quant_fp8_tensor:
        round to nearest even, codes 0x00..0x7E, -0 stored as +0)."""
        torch = self.torch
        if self.kind == "fp8":
            amax = float(w.abs().max()) or 1.0
            s = torch.tensor([2.0 ** np.ceil(np.log2(amax / 448.0))], dtype=torch.float32,
                             device=self.dev)
            code = (w / s).to(torch.float8_e4m3fn).view(torch.uint8)
            code = torch.where(code == 0x80, torch.zeros_like(code), code)
            return code.contiguous(), s
        amax = w.abs().amax(dim=1).clamp_min(1e-30)
        s = torch.exp2(torch.ceil(torch.log2(amax / 127.0)))
        q = torch.round(w / s[:, None]).clamp_(-127, 127).to(torch.int8)
        return q, s.to(torch.float32).contiguous()

    def bf16(self, t):
        return t.to(self.torch.bfloat16).contiguous()

    def generate(self, sink):
        """Call sink(kind, layer, name, tensor, scale) for every tensor, one
        at a time (so only one fp32 matrix is alive)."""
        cfg = self.cfg
        shapes = mat_shapes(cfg)
        emb = self.bf16(self._normal((cfg.vocab_size, cfg.dim), 0.02))
        sink("emb", -1, "emb", emb, None)
        del emb
        for i in range(cfg.n_layers):
            for n in MATS:
                q, s = self.quant(self._normal(shapes[n], 0.02))
                sink("mat", i, n, q, s)
                del q, s
            for n in ("attention_norm", "ffn_norm"):
                sink("norm", i, n, self.bf16(1.0 + self._normal((cfg.dim,), 0.1)), None)
        sink("norm", -1, "final_norm", self.bf16(1.0 + self._normal((cfg.dim,), 0.1)), None)
        q, s = self.quant(self._normal((cfg.vocab_size, cfg.dim), 0.02))
        sink("mat", -1, "lm", q, s)

    def bf16_weights(self):
        """Host BF16 copies of q * scale (exact) for the reference's path."""
        torch = self.torch
        out = {"layers": [dict() for _ in range(self.cfg.n_layers)]}

        def host_bf16(t):
            return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

        def sink(kind, layer, name, t, s):
            if kind == "mat":
                w = (t.view(torch.float8_e4m3fn).to(torch.float32) if self.kind == "fp8"
                     else t.to(torch.float32))
                v = host_bf16((w * s[:, None]).to(torch.bfloat16))
            else:
                v = host_bf16(t)
            if layer < 0:
                out[name] = v
            else:
                out["layers"][layer][name] = v

        self.torch.manual_seed(0)
        self._g.manual_seed(self.seed)
        self.generate(sink)
        return out
