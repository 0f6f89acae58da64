"""Documents why deep end-to-end parity must be layer-wise: in the reference numerics the
synthetic random-weight model amplifies a single fp16 ulp of input perturbation to percent-level
differences within a few layers (CPU oracle only)."""
import numpy as np

import dfssm_oracle as O
from dfssm_b200 import synthetic


def test_one_ulp_perturbation_grows_with_depth():
    w = synthetic.make_weights(synthetic.make_dims("tiny", 6), seed=0)
    a = O.OracleModel(w, 1, state_dtype="f32", emb="int8")
    b = O.OracleModel(w, 1, state_dtype="f32", emb="int8")
    x = a.E16[[123]]
    xa, xb = x.copy(), x.copy()
    xb[0, 7] = np.nextafter(xb[0, 7], np.float16(10))
    rel = []
    for l in range(6):
        xa, xb = a.layer(xa, l), b.layer(xb, l)
        rel.append(float(np.abs(xa.astype(np.float32) - xb.astype(np.float32)).max() / np.abs(xa).max()))
    # one ulp (~5e-4 relative in one of 256 inputs) becomes a >0.5% change of the residual stream
    assert rel[-1] > 5e-3, rel
