"""Sampling without a GPU: the device's uniform draw (pb_sample_uniform, a
host-callable function of the library) equals the oracle's restatement of
splitmix64, and the oracle's sample() follows llama-streaming.js:868-894
on hand-checked cases."""
import math

import numpy as np


def test_uniform_draw_matches_oracle(native, oracle):
    L = native.lib()
    for seed in (0, 1, 7, 2 ** 63 + 5, 2 ** 64 - 1):
        for ctr in (0, 1, 2, 1000, 2 ** 40):
            u = L.pb_sample_uniform(seed, ctr)
            assert u == oracle.sample_uniform(seed, ctr)
            assert 0.0 <= u < 1.0
    # splitmix64 published first output for state 0 (z after one gamma step)
    z = 0x9E3779B97F4A7C15
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & (2 ** 64 - 1)
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & (2 ** 64 - 1)
    z ^= z >> 31
    assert z == 0xE220A8397B1DCDAF
    assert L.pb_sample_uniform(0, 0) == (z >> 11) / 2.0 ** 53


def test_oracle_sample_rules(oracle):
    lg = np.array([0.5, 2.0, -1.0, 2.0, 1.0, np.nan, -np.inf], np.float32)
    # topK 1 is argmax with ties to the lower index; NaN never ranks
    assert oracle.sample(lg, 1, 0.8, 0.999) == 1
    # r = 0 always returns the top item; r just below 1 the last of the top K
    assert oracle.sample(lg, 3, 1.0, 0.0) == 1
    assert oracle.sample(lg, 3, 1.0, 0.9999999) == 4
    # the cumulative boundary: two equal tops share 1/(2+e^-1) each
    p0 = 1.0 / (2.0 + math.exp(-1.0))
    assert oracle.sample(lg, 3, 1.0, p0 * 0.999) == 1
    assert oracle.sample(lg, 3, 1.0, p0 * 1.001) == 3
    # temperature sharpens: at T = 0.01 the two tops take everything
    assert oracle.sample(lg, 7, 0.01, 0.9999) == 3
    # topK beyond the vocabulary keeps every non-NaN entry: near r = 1 the last
    # finite one (-1.0 at index 2) is drawn; -inf has probability 0
    assert oracle.sample(lg, 100, 1.0, 0.9999999) == 2
