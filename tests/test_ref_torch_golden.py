"""Pins oracle/ref_torch.py (the reference GPU driver restated in torch, used by the GPU parity
tests on CUDA) to golden vectors that the reference's own DFSSMModel produced
(tests/golden/make_golden.py).  On the CPU both run the same torch operations in the same order,
so tokens, logits, SSM and conv state must agree bit for bit."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import ref_torch as R  # noqa: E402
from dfssm_b200 import synthetic  # noqa: E402

HERE = os.path.join(os.path.dirname(__file__), "golden")
CASES = {"tiny": ("tiny", 2, 2, 12), "cfg0": ("1.3b", 2, 1, 8)}


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("variant", ["f16state", "f32state"])
def test_ref_torch_reproduces_reference_golden_bit_exact(name, variant):
    shape, nl, B, steps = CASES[name]
    g = np.load(os.path.join(HERE, f"golden_{name}.npz"))
    d = synthetic.make_dims(shape, nl)
    w = synthetic.make_weights(d, seed=0)
    torch.set_num_threads(4)  # the thread count the goldens were made with
    seen = []
    m = R.RefTorchModel(w, B, "cpu", torch.float16 if variant == "f16state" else torch.float32, "torch")
    m.spy = lambda name, a, b=None: seen.append((a.clone(), b.clone())) if name == "int_mm" and not seen else None
    toks, logs = m.generate(g["prompts"], steps)
    np.testing.assert_array_equal(toks, g[f"{variant}_tokens"])
    np.testing.assert_array_equal(seen[0][0].numpy(), g[f"{variant}_mm0_in"])
    np.testing.assert_array_equal(seen[0][1].numpy(), g[f"{variant}_mm0_out"])
    lg = logs.numpy()
    if f"{variant}_logits" in g:
        np.testing.assert_array_equal(lg, g[f"{variant}_logits"])
    else:
        np.testing.assert_array_equal(lg[..., :256], g[f"{variant}_logits_head"])
        np.testing.assert_array_equal(np.take_along_axis(lg, g[f"{variant}_top_idx"], -1), g[f"{variant}_top_val"])
    for l in range(nl):
        np.testing.assert_array_equal(m.h_states[l][:, :2].float().numpy(), g[f"{variant}_h{l}"])
        np.testing.assert_array_equal(m.h_states[l].double().sum(dim=(2, 3)).numpy(), g[f"{variant}_hsum{l}"])
        np.testing.assert_array_equal(m.conv_states[l].float().numpy(), g[f"{variant}_conv{l}"])
