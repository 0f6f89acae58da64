"""CPU checks of the oracle's restatement of the reference's sampling rule (eval/gen_test.py:69-87),
which the GPU sampling epilogue is tested against."""
import numpy as np

import dfssm_oracle as O


def test_nucleus_keeps_tokens_whose_preceding_mass_is_within_top_p():
    logits = np.log(np.array([0.5, 0.3, 0.15, 0.05], np.float32))
    seen = np.zeros(4, bool)
    for top_p, n in ((0.0, 1), (0.49, 1), (0.51, 2), (0.79, 2), (0.81, 3), (0.96, 4), (1.0, 4)):
        kept, p, mass = O.sample_nucleus(logits, seen, 1.0, top_p, 1.0)
        assert len(kept) == n, (top_p, kept)
        assert kept.tolist() == list(range(n))
        np.testing.assert_allclose(mass, p[:n].sum())


def test_repetition_penalty_divides_the_logit_whatever_its_sign():
    logits = np.array([-1.0, -2.0, 3.0], np.float32)
    seen = np.array([False, True, True])
    _, p, _ = O.sample_nucleus(logits, seen, 1.0, 1.0, 2.0)
    ref = np.exp(np.array([-1.0, -1.0, 1.5]) - 1.5)
    np.testing.assert_allclose(p, ref / ref.sum(), rtol=1e-6)


def test_temperature_scales_before_the_penalty():
    logits = np.array([2.0, 1.0], np.float32)
    _, p, _ = O.sample_nucleus(logits, np.array([True, False]), 0.5, 1.0, 4.0)
    ref = np.exp(np.array([1.0, 2.0]) - 2.0)
    np.testing.assert_allclose(p, ref / ref.sum(), rtol=1e-6)
