"""The numpy oracle reproduces the reference sampler's token ids.

``tests/golden/golden.json`` holds ids produced by QEdge's own
``BatchSampler`` (``src/compute/sampler.py:25-41``) under the shared-noise
adapter; this pins ``oracle/sampler_oracle.py`` before it is trusted as the
checker for the CUDA kernel.
"""
import numpy as np
import pytest

from oracle import sampler_oracle as O
from tests.golden import cases as C

CASES = C.build_cases()


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name, golden):
    w, spec = CASES[name]
    g = golden["cases"][name]
    assert C.digest(w.logits_bits) == g["logits_sha256"], "input generator drifted"
    noise = C.make_noise(spec, w.B, w.V)
    assert C.digest(noise) == g["noise_sha256"], "noise generator drifted"
    ids = O.sample(w.logits_f32(), w.temperatures, w.top_ps, noise,
                   rep_penalties=w.rep_penalties, history=w.history,
                   history_lens=w.history_lens, all_greedy=g["all_greedy"],
                   use_top_p=w.use_top_p)
    np.testing.assert_array_equal(ids, np.asarray(g["ids"], dtype=np.int64))


def test_multinomial_is_exponential_race(golden):
    assert golden["multinomial_is_exponential_race"]
