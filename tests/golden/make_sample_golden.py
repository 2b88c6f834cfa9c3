"""Generate tests/golden/sample_vectors.npz: the reference's own top-p
sampler (sample_top_p, src/compute/sampler_topp.c:113, built into
oracle/_ref) on seeded logits, after the server's repetition penalty and UNK
block (src/server/worker.c:436-444), restated here in float32 numpy.

    python tests/golden/make_sample_golden.py

The cases (logits before the penalty, token history, temperature, top_p,
rand() seed) are regenerated from numpy seed 47 by cases(); the file keeps,
per case, the draw the reference takes (rand() / RAND_MAX after
srand(seed)), the token it returns and the first 8 bytes of the logits (a
check that the regenerated inputs are the ones used).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

PENALTY = np.float32(1.2)  # REPETITION_PENALTY, src/config.h:62


def penalise(lg, hist):
    lg = lg.copy()
    for t in hist:
        lg[t] = lg[t] / PENALTY if lg[t] > 0 else lg[t] * PENALTY
    lg[0] = np.float32(-1e9)
    return lg


SHAPES = [(32000, 3.0, 0.7, 0.9), (32000, 1.0, 0.7, 0.9), (32000, 6.0, 1.0, 0.5),
          (128256, 4.0, 0.7, 0.9), (1000, 2.0, 1.3, 1.0), (1000, 8.0, 0.2, 0.9)]
PER_SHAPE = 8


def cases():
    """(logits, history, temperature, top_p, rand seed) per case, all from
    numpy seed 47: the tests regenerate them from here instead of storing
    megabytes of logits."""
    r = np.random.default_rng(47)
    out = []
    for n, scale, temp, top_p in SHAPES:
        for _ in range(PER_SHAPE):
            lg = (scale * r.standard_normal(n)).astype(np.float32)
            hist = r.integers(0, n, size=int(r.integers(0, 300))).astype(np.int32)
            out.append((lg, hist, np.float32(temp), np.float32(top_p),
                        int(r.integers(1, 2**31 - 1))))
    return out


def main():
    R = O.ref()
    draws, toks, digests = [], [], []
    for lg, hist, temp, top_p, seed in cases():
        pl = penalise(lg, hist)
        draws.append(R.refd_first_rand(seed))
        toks.append(R.refd_sample_top_p(pl, pl.size, temp, top_p, seed))
        digests.append(int.from_bytes(lg[:64].tobytes()[:8], "little"))
    np.savez_compressed(
        os.path.join(HERE, "sample_vectors.npz"),
        draw=np.array(draws, np.float32), token=np.array(toks, np.int32),
        logits_head=np.array(digests, np.uint64), penalty=PENALTY)


if __name__ == "__main__":
    main()
