"""Device-generated weights (vx_model_create_synth, vxc_synth.cu) against the
GGUF the library's writer makes for the same configuration and seed: the
forward logits of the two models agree to 1e-5 x max|logit|.  The integer
and fp32 steps of the generator are the writer's; only the double-precision
log/sqrt/cos/sin of the Box-Muller step are the device's, which can move a
weight by one quantisation step in rare boundary cases."""
import numpy as np
import pytest

import fixtures

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["tiny_target", "tiny_draft", "l7b_2layer"])
def test_synth_model_matches_written_checkpoint(cuda, name):
    import vxb200
    e, L, h, kv, ff, v, wt, seed, th = fixtures.CONFIGS[name]
    a = vxb200.Model(fixtures.path(name))
    b = vxb200.Model(None, synth=(e, L, h, kv, ff, v, wt, seed, th))
    toks = np.random.default_rng(31).integers(0, v, 12).astype(np.int32)
    for chunk in (toks[:9], toks[9:10], toks[10:]):
        la, lb = a.forward(chunk), b.forward(chunk)
        assert float(np.max(np.abs(la - lb))) <= 1e-5 * float(np.max(np.abs(la)))
    a.close()
    b.close()
