"""The synthetic router logits (routing.logits) are the ones routes() selects
from: for the softmax schemes the top-k of the logits, in descending order,
are routes()'s ids for every token and layer."""
import numpy as np


def test_logits_select_the_routes(gxlib):
    from galactus_b200.routing import logits, routes
    for name in ("qwen3-30b", "olmoe"):
        m = gxlib.MODELS[name]
        lg = logits(m, 6, 3, seed=7, rho=0.7)
        ids, w = routes(m, 6, 3, seed=7, rho=0.7)
        assert lg.shape == (6, 3, m.experts) and lg.dtype == np.float32
        top = np.argsort(-lg, axis=2, kind="stable")[:, :, :m.used]
        np.testing.assert_array_equal(top, ids)
        assert np.all(w > 0)
