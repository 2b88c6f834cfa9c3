"""Host-side integer logic of the tensor-core GEMM (csrc/tc_gemm.cu), on CPU.

1. Stream-K split: CTA i of G owns units [i*W/G, (i+1)*W/G); the combine
   finds the CTA holding unit u as ((u+1)*G + W - 1)/W - 1.  Checked against
   a brute-force search for many (W, G).
2. Digit planes: x' = rint(x * 2080768 / max|x|) = d0*2^14 + d1*2^7 + d2 with
   d0 in [-127, 127] and d1, d2 in [-64, 64] (signed INT8 operands whose
   products with INT8 weights accumulate exactly in int32 up to K = 28672),
   reconstructing x' exactly.
"""
import numpy as np

FULL = 2080768  # 127 * 2^14


def unit_start(i, W, G):
    return i * W // G


def holder(u, W, G):
    return ((u + 1) * G + W - 1) // W - 1


def test_stream_k_holder_formula():
    rng = np.random.default_rng(0)
    cases = [(1024, 148), (7168, 148), (32064, 148), (112, 112), (8, 8), (10, 4), (3584, 148)]
    cases += [(int(rng.integers(1, 5000)), int(rng.integers(1, 200))) for _ in range(200)]
    for W, G in cases:
        G = min(G, W)  # the launch uses min(grid, W) CTAs
        starts = [unit_start(i, W, G) for i in range(G + 1)]
        assert all(starts[i + 1] > starts[i] for i in range(G)), (W, G)  # no empty CTA
        for u in {0, W - 1, W // 2, W // 3} | set(rng.integers(0, W, 20).tolist()):
            i = holder(u, W, G)
            assert starts[i] <= u < starts[i + 1], (W, G, u, i)


def digits(xv):
    d0 = np.rint(xv / 16384.0).astype(np.int64)
    r0 = xv - d0 * 16384
    d1 = np.rint(r0 / 128.0).astype(np.int64)
    d2 = r0 - d1 * 128
    return d0, d1, d2


def test_digit_planes_exact_and_in_range():
    rng = np.random.default_rng(1)
    for scale in (1e-3, 1.0, 37.0):
        x = (rng.standard_normal(4096) * scale).astype(np.float32)
        x[:3] = [0.0, np.abs(x).max(), -np.abs(x).max()]
        mx = np.float32(np.abs(x).max())
        xv = np.rint(x.astype(np.float64) * (FULL / np.float64(mx))).astype(np.int64)
        d0, d1, d2 = digits(xv)
        assert np.array_equal(d0 * 16384 + d1 * 128 + d2, xv)
        assert d0.min() >= -127 and d0.max() <= 127
        assert np.abs(d1).max() <= 64 and np.abs(d2).max() <= 64
        # relative rounding error of each element against the row's max
        err = np.abs(xv * (np.float64(mx) / FULL) - x.astype(np.float64)).max()
        assert err <= 0.5 * float(mx) / FULL * (1 + 1e-12)
    # int32 accumulation bound at the largest K of the shapes (28672)
    assert 127 * 127 * 28672 < 2 ** 31
